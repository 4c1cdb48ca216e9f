// .ltq tile packing and spec decode on the device (lumen-inference/ltq-research src/ltq_file.py:54-148, tile fields of
// src/ltq_format.py:104-147).
//
// A row slice [R, K] (R, K multiples of 16) is T = (R / 16) (K / 16) tiles of 16 x 16, ordered by row group then by
// 16-column block; position t = 16 r + c inside a tile.  Per tile the fields are u16 words:
//   codes  16 words           bit c of word r = label(r, c) & 1
//   planes (K - 2) x 16 words plane p - 1: bit c of word r = bit p of u(r, c)
//   lsb    16 / 8 / 12 words  bit 0 of u at every position / at even positions (D2) / at the first three positions of
//                             each group of four (D4), bits numbered in position order
//   gains  ceil(256 / sub * h / 16) words: the h-bit gain index of each sub-block, LSB first
// and the slice stores them as four structure-of-arrays regions [T][words], each starting at a multiple of 64 bytes
// (the padding goes before every region, empty ones included).
//
// ltq_pack_slice_kernel / ltq_decode_slice_kernel: one warp per tile, a grid of 4 CTAs per SM walking the tiles.  Lane L
// owns row L / 2, columns 8 (L & 1) .. + 7 (one 16-byte load of idx, one 8-byte load of gi); a field word is assembled
// from the owning lanes' bit fragments with warp shuffles and reductions.  Both are HBM-bound (3 bytes read per weight
// for packing, tile_bytes / 256 written; the verify decode reads the packed tile and the 4-byte reference value).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "ltq_b200.h"
#include "stride_grid.cuh"

namespace {

constexpr unsigned FULL = 0xffffffffu;

struct SliceLayout {
    int nw[4];          // words per tile of each region
    long long off[4];   // byte offset of each region
    long long total;    // slice bytes
};

SliceLayout slice_layout(long long T, int kbits, int frac, int h, int sub)
{
    SliceLayout L;
    L.nw[0] = 16;
    L.nw[1] = 16 * (kbits - 2);
    L.nw[2] = frac == 0 ? 16 : (frac == 1 ? 8 : 12);
    L.nw[3] = (256 / sub * h + 15) / 16;
    long long o = 0;
    for (int r = 0; r < 4; r++) {
        o = (o + 63) / 64 * 64;
        L.off[r] = o;
        o += 2 * T * L.nw[r];
    }
    L.total = o;
    return L;
}

struct PackArgs {
    int kbits, frac, h, sub, tiles_per_row;  // tiles_per_row = K / 16
    long long T;
    int nw[4];
    long long off[4];
};

// Word w (< 32 lanes' worth) of a bit string in which lane l holds the nb bits [nb l, nb l + nb): every lane calls
// with its own w; lanes whose w is out of range get garbage they do not store.
__device__ __forceinline__ uint32_t gather_word(uint32_t v, int nb, int w)
{
    const int l0 = (16 * w) / nb;
    const int nsrc = 16 / nb + 1;
    uint32_t word = 0;
    for (int k = 0; k <= nsrc; k++) {
        const int src = l0 + k;
        const uint32_t x = __shfl_sync(FULL, v, src & 31);
        const int sh = nb * src - 16 * w;
        if (src < 32 && sh < 16 && sh > -nb) word |= sh >= 0 ? (x << sh) : (x >> (-sh));
    }
    return word & 0xffffu;
}

// zeros in the padding before regions 1..3 (less than 64 bytes each), by the first 64 threads of CTA 0
__device__ __forceinline__ void zero_gaps(uint8_t* out, const PackArgs& a)
{
    if (blockIdx.x != 0 || threadIdx.x >= 64) return;
    for (int rr = 1; rr < 4; rr++) {
        const long long lo = a.off[rr - 1] + 2 * a.T * a.nw[rr - 1];
        if (lo + threadIdx.x < a.off[rr]) out[lo + threadIdx.x] = 0;
    }
}

// Grid-stride over tiles, one warp per tile; the next tile's idx / gi loads are issued before the current tile's
// fields are built.  Byte-aligned fields (codes, planes, lsb of FRAC 0): lane 2r holds bits 0..7 of word r and lane
// 2r + 1 bits 8..15, so one shuffle joins them (four fields per 32-bit exchange).  Gain indices: an OR-reduction of
// the h-bit values at bit h k over the warp.  Every byte of the slice is written (fields by the tiles' warps, padding
// by zero_gaps), so the output needs no clearing first.
template <int KB>
__global__ void __launch_bounds__(256, 4) ltq_pack_slice_kernel(const int16_t* __restrict__ idx,
                                                             const uint8_t* __restrict__ gi, long long ld,
                                                             uint8_t* __restrict__ out, const PackArgs a)
{
    constexpr int U = 1 << (KB - 1), NPL = KB - 2;
    zero_gaps(out, a);
    const int lane = threadIdx.x & 31, r = lane >> 1, hf = lane & 1;
    const long long step = (long long)gridDim.x * (blockDim.x >> 5);
    long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.T) return;
    auto src = [&](long long tt) { return (tt / a.tiles_per_row * 16 + r) * ld + tt % a.tiles_per_row * 16 + 8 * hf; };
    long long base = src(t);
    uint4 niv = *reinterpret_cast<const uint4*>(idx + base);
    uint2 ngv = *reinterpret_cast<const uint2*>(gi + base);
    const int nsb = 256 / a.sub;
    for (; t < a.T; t += step) {
        const uint4 iv = niv;
        const uint2 gv = ngv;
        if (t + step < a.T) {
            base = src(t + step);
            niv = *reinterpret_cast<const uint4*>(idx + base);
            ngv = *reinterpret_cast<const uint2*>(gi + base);
        }
        const uint32_t iw[4] = {iv.x, iv.y, iv.z, iv.w};
        uint32_t cb = 0, lsb = 0, pl[NPL > 0 ? NPL : 1];
#pragma unroll
        for (int p = 0; p < (NPL > 0 ? NPL : 1); p++) pl[p] = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t v = (iw[j >> 1] >> (16 * (j & 1))) & 0xffffu;
            const uint32_t lab = v >> (KB - 1), u = v & (U - 1);
            cb |= (lab & 1u) << j;
            lsb |= (u & 1u) << j;
#pragma unroll
            for (int p = 0; p < NPL; p++) pl[p] |= ((u >> (p + 1)) & 1u) << j;
        }
        // bytes: [codes, lsb (FRAC 0), plane 1, plane 2], [planes 3..6]
        const uint32_t f0 = cb | (lsb << 8) | (NPL > 0 ? pl[0] << 16 : 0u) | (NPL > 1 ? pl[NPL > 1 ? 1 : 0] << 24 : 0u);
        const uint32_t o0 = __shfl_down_sync(FULL, f0, 1);
        uint32_t f1 = 0, o1 = 0;
        if constexpr (NPL > 2) {
#pragma unroll
            for (int p = 2; p < NPL; p++) f1 |= pl[p] << (8 * (p - 2));
            o1 = __shfl_down_sync(FULL, f1, 1);
        }
        uint16_t* reg0 = reinterpret_cast<uint16_t*>(out + a.off[0]) + t * a.nw[0];
        uint16_t* reg1 = reinterpret_cast<uint16_t*>(out + a.off[1]) + t * a.nw[1];
        uint16_t* reg2 = reinterpret_cast<uint16_t*>(out + a.off[2]) + t * a.nw[2];
        if (!hf) {
            reg0[r] = (uint16_t)__byte_perm(f0, o0, 0x40);
            if (NPL > 0) reg1[r] = (uint16_t)__byte_perm(f0, o0, 0x62);
            if (NPL > 1) reg1[16 + r] = (uint16_t)__byte_perm(f0, o0, 0x73);
#pragma unroll
            for (int p = 2; p < NPL; p++) reg1[16 * p + r] = (uint16_t)__byte_perm(f1, o1, (p - 2) | ((p + 2) << 4));
            if (a.frac == 0) reg2[r] = (uint16_t)__byte_perm(f0, o0, 0x51);
        }
        // lsb of the parity modes: 4 bits a lane (D2, the even positions) or 6 (D4, the first three of each quad)
        if (a.frac == 1) {
            const uint32_t lv = (lsb & 1) | ((lsb >> 1) & 2) | ((lsb >> 2) & 4) | ((lsb >> 3) & 8);
            uint32_t x = lv | (__shfl_down_sync(FULL, lv, 1) << 4);
            x |= __shfl_down_sync(FULL, x, 2) << 8;
            if ((lane & 3) == 0) reg2[lane >> 2] = (uint16_t)x;
        } else if (a.frac == 2) {
            const uint32_t lv = (lsb & 7) | (((lsb >> 4) & 7) << 3);
            const uint32_t lw = gather_word(lv, 6, lane);
            if (lane < a.nw[2]) reg2[lane] = (uint16_t)lw;
        }
        // gains: the index at the first position of sub-block k (row k sub / 16, column 0: lane 2 (k sub / 16),
        // element 0) goes to bit h k of a 64-bit string (16 sub-blocks x 4 bits at most)
        if (a.h > 0) {
            const uint32_t gk = __shfl_sync(FULL, gv.x & 0xffu, (2 * ((lane * a.sub) >> 4)) & 31) & ((1u << a.h) - 1u);
            const int b = a.h * lane;
            uint32_t lo = 0, hi = 0;
            if (lane < nsb) {
                if (b < 32) {
                    lo = gk << b;
                    if (b + a.h > 32) hi = gk >> (32 - b);
                } else {
                    hi = gk << (b - 32);
                }
            }
            lo = __reduce_or_sync(FULL, lo);
            hi = __reduce_or_sync(FULL, hi);
            uint16_t* reg3 = reinterpret_cast<uint16_t*>(out + a.off[3]) + t * a.nw[3];
            if (lane < a.nw[3]) reg3[lane] = (uint16_t)((lane < 2 ? lo : hi) >> (16 * (lane & 1)));
        }
    }
}

struct DecodeArgs {
    PackArgs p;
    unsigned m0, m1, m2;
    int nmask;
    int vec_out, vec_ref;  // 16-byte aligned rows: float4 stores / loads
};

// Grid-stride over tiles, one warp per tile; lane L owns row L / 2 and columns 8 (L & 1) .. + 7.  The ten code bits
// ending at a position are one funnel shift of two words of the tile's 256-bit code string (the string wraps around:
// tail-biting) and a bit reversal; label bits from the masks' parities; the value table and gains from shared memory.
template <int KB, int FRAC>
__global__ void __launch_bounds__(256, 4) ltq_decode_slice_kernel(const uint8_t* __restrict__ data,
                                                               const float* __restrict__ lut,
                                                               const float* __restrict__ gain_tab,
                                                               float* __restrict__ out, long long ld_out,
                                                               const float* __restrict__ ref, long long ld_ref,
                                                               unsigned long long* __restrict__ mismatches,
                                                               const DecodeArgs d)
{
    constexpr int U = 1 << (KB - 1);
    __shared__ float s_lut[16 * 128];
    __shared__ float s_gain[16];
    const PackArgs& a = d.p;
    for (int i = threadIdx.x; i < (2 << d.nmask) * U; i += blockDim.x) s_lut[i] = lut[i];
    if (a.h > 0 && threadIdx.x < (1 << a.h)) s_gain[threadIdx.x] = gain_tab[threadIdx.x];
    __syncthreads();
    const int lane = threadIdx.x & 31, r = lane >> 1, hf = lane & 1;
    const int w_hi = r >> 1, w_lo = (w_hi + 7) & 7;  // 32-bit code words holding this lane's positions and the 32 before
    const int o0 = 16 * (r & 1) + 8 * hf;            // bit offset of the lane's first position in word w_hi
    const int lb0 = FRAC == 0 ? 16 * r + 8 * hf : (FRAC == 1 ? 8 * r + 4 * hf : 12 * r + 6 * hf);
    const int lw0 = lb0 >> 4, lsh = lb0 & 15;
    const int gb0 = (16 * r / a.sub) * a.h;
    const int gw0 = gb0 >> 4, gsh = gb0 & 15;
    const unsigned gmask = (1u << a.h) - 1u;
    const long long step = (long long)gridDim.x * (blockDim.x >> 5);
    unsigned bad = 0;
    for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.T; t += step) {
        const long long rg = t / a.tiles_per_row, kb = t % a.tiles_per_row;
        const uint32_t* cw = reinterpret_cast<const uint32_t*>(data + a.off[0] + t * 32);
        const uint32_t hi = __ldg(cw + w_hi), lo = __ldg(cw + w_lo);
        const uint16_t* pl = reinterpret_cast<const uint16_t*>(data + a.off[1]) + t * a.nw[1];
        const uint16_t* lw = reinterpret_cast<const uint16_t*>(data + a.off[2]) + t * a.nw[2];
        const uint16_t* gw = reinterpret_cast<const uint16_t*>(data + a.off[3]) + t * a.nw[3];
        uint32_t pw[KB > 2 ? KB - 2 : 1];
#pragma unroll
        for (int p = 0; p < KB - 2; p++) pw[p] = (uint32_t)__ldg(pl + p * 16 + r) >> (8 * hf);
        uint32_t lsb = (uint32_t)__ldg(lw + lw0);
        if (FRAC == 2 && lw0 + 1 < a.nw[2]) lsb |= (uint32_t)__ldg(lw + lw0 + 1) << 16;
        lsb >>= lsh;
        float gain = 1.0f;
        if (a.h > 0) {
            uint32_t gv = (uint32_t)__ldg(gw + gw0);
            if (gsh + a.h > 16 && gw0 + 1 < a.nw[3]) gv |= (uint32_t)__ldg(gw + gw0 + 1) << 16;
            gain = s_gain[(gv >> gsh) & gmask];
        }
        const long long col = kb * 16 + 8 * hf;
        float rv[8];
        if (ref) {
            const float* rrow = ref + (rg * 16 + r) * ld_ref + col;
            if (d.vec_ref) {
                const float4 x0 = __ldcs(reinterpret_cast<const float4*>(rrow));
                const float4 x1 = __ldcs(reinterpret_cast<const float4*>(rrow) + 1);
                rv[0] = x0.x; rv[1] = x0.y; rv[2] = x0.z; rv[3] = x0.w; rv[4] = x1.x; rv[5] = x1.y; rv[6] = x1.z; rv[7] = x1.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) rv[j] = rrow[j];
            }
        }
        float val[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t win = __funnelshift_rc(lo, hi, o0 + j + 1);
            const unsigned st = __brev(win) & 0x3ffu;
            const unsigned v = st >> 1;
            const int lab = (int)(st & 1) | ((__popc(v & d.m0) & 1) << 1) | ((__popc(v & d.m1) & 1) << 2) |
                            ((__popc(v & d.m2) & 1) << 3);
            int u;
            if (FRAC == 0) {
                u = (lsb >> j) & 1;
            } else if (FRAC == 1) {
                u = (lsb >> (j >> 1)) & 1;
            } else {
                const uint32_t q = lsb >> (3 * (j >> 2));
                u = (j & 3) < 3 ? (int)((q >> (j & 3)) & 1) : (int)((q ^ (q >> 1) ^ (q >> 2)) & 1);
            }
#pragma unroll
            for (int p = 0; p < KB - 2; p++) u |= (int)((pw[p] >> j) & 1) << (p + 1);
            val[j] = __fmul_rn(gain, s_lut[lab * U + u]);
            if (ref && val[j] != rv[j]) bad++;
        }
        if (out) {
            float* orow = out + (rg * 16 + r) * ld_out + col;
            if (d.vec_out) {
                reinterpret_cast<float4*>(orow)[0] = make_float4(val[0], val[1], val[2], val[3]);
                reinterpret_cast<float4*>(orow)[1] = make_float4(val[4], val[5], val[6], val[7]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) orow[j] = val[j];
            }
        }
    }
    if (mismatches) {
        for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(FULL, bad, o);
        if (lane == 0 && bad) atomicAdd(mismatches, (unsigned long long)bad);
    }
}

bool fmt_ok(int R, int K, int kbits, int frac, int h, int sub)
{
    return R >= 0 && K >= 0 && R % 16 == 0 && K % 16 == 0 && kbits >= 2 && kbits <= 8 && frac >= 0 && frac <= 2 &&
           h >= 0 && h <= 4 && (sub == 16 || sub == 32) && (frac != 2 || kbits >= 2);
}

PackArgs pack_args(int R, int K, int kbits, int frac, int h, int sub)
{
    PackArgs a{};
    a.kbits = kbits; a.frac = frac; a.h = h; a.sub = sub; a.tiles_per_row = K / 16;
    a.T = (long long)(R / 16) * (K / 16);
    const SliceLayout L = slice_layout(a.T, kbits, frac, h, sub);
    for (int i = 0; i < 4; i++) { a.nw[i] = L.nw[i]; a.off[i] = L.off[i]; }
    return a;
}


// ------------------------------------------------------------------------------------------------
// Batch-1 matrix-vector product straight from a packed slice (the inference-side step after quantization;
// src/cuda/ltq_matvec_bench.cu:77-150 prototypes it on a row-tile layout, this runs on the .ltq file's 16 x 16 tiles):
//   y[r] = sum_b d[r][b] * sum_{k in block b} val(r, k) * xr[k],   d[r][b] = d_row[r] * 2^(e[r][b] / 4)
// with val the spec-decoded tile value gain[g] * lut[label * U + u] and xr the rotated input H256 (suh * x), so that
// y = W x for the assembled W = H256(d val) * suh.  One CTA per 16-row tile group with one warp per 256-column block
// (at most 32, round-robin beyond), 64 registers a thread so that 32 warps fit an SM; lane L owns row L / 2 and columns
// 8 (L & 1) .. + 7 of every tile (as the decode kernel).  The
// ten code bits ending at a position are one funnel shift of the tile's 256-bit code string and a bit reversal.  Sums:
// per lane sequential fmas over a block's 16 tiles x 8 columns, the block scale, the two half-rows, then the warps in a
// fixed order — deterministic.
// ------------------------------------------------------------------------------------------------
template <int KB, int FRAC>
__global__ void __launch_bounds__(1024, 1) ltq_matvec_slice_kernel(const uint8_t* __restrict__ data,
                                                                   const float* __restrict__ lut,
                                                                   const float* __restrict__ gain_tab,
                                                                   const uint16_t* __restrict__ d_row,
                                                                   const int8_t* __restrict__ e, long long ld_e,
                                                                   const float* __restrict__ xr,
                                                                   float* __restrict__ y, const DecodeArgs d)
{
    constexpr int U = 1 << (KB - 1);
    __shared__ float red[32][16];
    __shared__ float s_lut[16 * 32];  // value table (labels x U <= 16 x 32) and gains, read per position
    __shared__ float s_gain[16];
    const PackArgs& a = d.p;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 1, hf = lane & 1;
    const long long rg = blockIdx.x;
    const long long row = rg * 16 + r;
    const int nblk = a.tiles_per_row / 16;
    const float drow = __half2float(__ushort_as_half(d_row[row]));
    for (int i = threadIdx.x; i < (2 << d.nmask) * U; i += blockDim.x) s_lut[i] = lut[i];
    if (a.h > 0 && threadIdx.x < (1 << a.h)) s_gain[threadIdx.x] = gain_tab[threadIdx.x];
    __syncthreads();
    const int w_hi = r >> 1, w_lo = (w_hi + 7) & 7;  // 32-bit code words holding this lane's positions and the 32 before
    const int o0 = 16 * (r & 1) + 8 * hf;            // bit offset of the lane's first position in word w_hi
    // the lane's low-bit field: FRAC 0 one bit per position (word r), D2 one per pair (word r / 2), D4 three per quad
    // (6 bits from bit 12 r + 6 hf, possibly across two words)
    const int lb0 = FRAC == 0 ? 16 * r + 8 * hf : (FRAC == 1 ? 8 * r + 4 * hf : 12 * r + 6 * hf);
    const int lw0 = lb0 >> 4, lsh = lb0 & 15;
    const int gb0 = (16 * r / a.sub) * a.h;           // the sub-block's gain-index bits
    const int gw0 = gb0 >> 4, gsh = gb0 & 15;
    const unsigned gmask = (1u << a.h) - 1u;
    const int nwarps = blockDim.x >> 5;
    float acc = 0.f;
    for (int b = warp; b < nblk; b += nwarps) {
        float part = 0.f;
        for (int kt = 0; kt < 16; kt++) {
            const long long t = rg * a.tiles_per_row + (long long)b * 16 + kt;
            const uint32_t* cw = reinterpret_cast<const uint32_t*>(data + a.off[0] + t * 32);
            const uint32_t hi = __ldg(cw + w_hi), lo = __ldg(cw + w_lo);
            const uint16_t* pl = reinterpret_cast<const uint16_t*>(data + a.off[1]) + t * a.nw[1];
            const uint16_t* lw = reinterpret_cast<const uint16_t*>(data + a.off[2]) + t * a.nw[2];
            const uint16_t* gw = reinterpret_cast<const uint16_t*>(data + a.off[3]) + t * a.nw[3];
            uint32_t pw[KB > 2 ? KB - 2 : 1];  // plane p - 1 at the lane's 8 columns
#pragma unroll
            for (int p = 0; p < KB - 2; p++) pw[p] = (uint32_t)__ldg(pl + p * 16 + r) >> (8 * hf);
            uint32_t lsb = (uint32_t)__ldg(lw + lw0);
            if (FRAC == 2 && lw0 + 1 < a.nw[2]) lsb |= (uint32_t)__ldg(lw + lw0 + 1) << 16;
            lsb >>= lsh;
            float gain = 1.0f;
            if (a.h > 0) {
                uint32_t gv = (uint32_t)__ldg(gw + gw0);
                if (gsh + a.h > 16 && gw0 + 1 < a.nw[3]) gv |= (uint32_t)__ldg(gw + gw0 + 1) << 16;
                gain = s_gain[(gv >> gsh) & gmask];
            }
            const float* xt = xr + (long long)b * 256 + kt * 16 + 8 * hf;
            const float4 xa = __ldg(reinterpret_cast<const float4*>(xt)), xb = __ldg(reinterpret_cast<const float4*>(xt + 4));
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                // bits pos - 31 .. pos of the code string, newest in bit 31; reversed, the state s has the newest in bit 0
                const uint32_t win = __funnelshift_rc(lo, hi, o0 + j + 1);
                const unsigned st = __brev(win) & 0x3ffu;
                const unsigned v = st >> 1;
                const int lab = (int)(st & 1) | ((__popc(v & d.m0) & 1) << 1) | ((__popc(v & d.m1) & 1) << 2) |
                                ((__popc(v & d.m2) & 1) << 3);
                int u;
                if (FRAC == 0) {
                    u = (lsb >> j) & 1;
                } else if (FRAC == 1) {
                    u = (lsb >> (j >> 1)) & 1;
                } else {
                    const uint32_t q = lsb >> (3 * (j >> 2));
                    u = (j & 3) < 3 ? (int)((q >> (j & 3)) & 1) : (int)((q ^ (q >> 1) ^ (q >> 2)) & 1);
                }
#pragma unroll
                for (int p = 0; p < KB - 2; p++) u |= (int)((pw[p] >> j) & 1) << (p + 1);
                const float val = __fmul_rn(gain, s_lut[lab * U + u]);
                part = __fmaf_rn(val, xv[j], part);
            }
        }
        const float db = __fmul_rn(drow, exp2f(0.25f * (float)e[row * ld_e + b]));
        acc = __fmaf_rn(db, part, acc);
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(FULL, acc, 1));
    if (hf == 0) red[warp][r] = acc;
    __syncthreads();
    if (threadIdx.x < 16) {
        float s = red[0][threadIdx.x];
        for (int w = 1; w < nwarps; w++) s = __fadd_rn(s, red[w][threadIdx.x]);
        y[rg * 16 + threadIdx.x] = s;
    }
}

template <int KB>
int launch_matvec_kb(int frac, unsigned grid, int threads, cudaStream_t st, const uint8_t* data, const float* lut,
                     const float* gain_tab, const uint16_t* d_row, const int8_t* e, long long ld_e, const float* x_rot,
                     float* y, const DecodeArgs& d)
{
    switch (frac) {
        case 0: ltq_matvec_slice_kernel<KB, 0><<<grid, threads, 0, st>>>(data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 1: ltq_matvec_slice_kernel<KB, 1><<<grid, threads, 0, st>>>(data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 2: ltq_matvec_slice_kernel<KB, 2><<<grid, threads, 0, st>>>(data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        default: return -1;
    }
    return 0;
}

template <int KB>
int launch_decode_kb(int frac, unsigned grid, cudaStream_t st, const uint8_t* data, const float* lut,
                     const float* gain_tab, float* out, long long ld_out, const float* ref, long long ld_ref,
                     unsigned long long* mismatches, const DecodeArgs& d)
{
    switch (frac) {
        case 0: ltq_decode_slice_kernel<KB, 0><<<grid, 256, 0, st>>>(data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 1: ltq_decode_slice_kernel<KB, 1><<<grid, 256, 0, st>>>(data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 2: ltq_decode_slice_kernel<KB, 2><<<grid, 256, 0, st>>>(data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        default: return -1;
    }
    return 0;
}

}  // namespace

extern "C" size_t ltq_slice_bytes(int R, int K, int kbits, int frac, int h, int sub)
{
    if (!fmt_ok(R, K, kbits, frac, h, sub)) return 0;
    return (size_t)slice_layout((long long)(R / 16) * (K / 16), kbits, frac, h, sub).total;
}

extern "C" int ltq_pack_slice(const int16_t* idx, const uint8_t* gi, long long ld, int R, int K, int kbits, int frac,
                              int h, int sub, uint8_t* out, size_t out_bytes, void* stream)
{
    if (!fmt_ok(R, K, kbits, frac, h, sub) || ld < K || (ld % 8) || ((uintptr_t)idx & 15) || ((uintptr_t)gi & 7) ||
        ((uintptr_t)out & 63))
        return -1;
    const PackArgs a = pack_args(R, K, kbits, frac, h, sub);
    if (out_bytes < (size_t)slice_layout(a.T, kbits, frac, h, sub).total) return -1;
    if (a.T == 0) return 0;
    const unsigned grid = (unsigned)stride_grid((a.T + 7) / 8, 4);
    const cudaStream_t st = (cudaStream_t)stream;
    switch (kbits) {
        case 2: ltq_pack_slice_kernel<2><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 3: ltq_pack_slice_kernel<3><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 4: ltq_pack_slice_kernel<4><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 5: ltq_pack_slice_kernel<5><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 6: ltq_pack_slice_kernel<6><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 7: ltq_pack_slice_kernel<7><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        case 8: ltq_pack_slice_kernel<8><<<grid, 256, 0, st>>>(idx, gi, ld, out, a); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

extern "C" int ltq_decode_slice(const uint8_t* data, int R, int K, int kbits, int frac, int h, int sub,
                                const int* masks, int n_masks, const float* lut, const float* gain_tab, float* out,
                                long long ld_out, const float* ref, long long ld_ref, unsigned long long* mismatches,
                                void* stream)
{
    if (!fmt_ok(R, K, kbits, frac, h, sub) || !masks || n_masks < 1 || n_masks > 3 || !lut || (h > 0 && !gain_tab) ||
        (out && ld_out < K) || (ref && ld_ref < K) || ((uintptr_t)data & 63))
        return -1;
    DecodeArgs d{};
    d.p = pack_args(R, K, kbits, frac, h, sub);
    d.m0 = (unsigned)masks[0];
    d.m1 = n_masks > 1 ? (unsigned)masks[1] : 0u;
    d.m2 = n_masks > 2 ? (unsigned)masks[2] : 0u;
    d.nmask = n_masks;
    d.vec_out = out && !((uintptr_t)out & 15) && !(ld_out & 3);
    d.vec_ref = ref && !((uintptr_t)ref & 15) && !(ld_ref & 3);
    if (d.p.T == 0) return 0;
    const unsigned grid = (unsigned)stride_grid((d.p.T + 7) / 8, 4);
    int rc = -1;
    switch (kbits) {
        case 2: rc = launch_decode_kb<2>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 3: rc = launch_decode_kb<3>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 4: rc = launch_decode_kb<4>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 5: rc = launch_decode_kb<5>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 6: rc = launch_decode_kb<6>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 7: rc = launch_decode_kb<7>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        case 8: rc = launch_decode_kb<8>(frac, grid, (cudaStream_t)stream, data, lut, gain_tab, out, ld_out, ref, ld_ref, mismatches, d); break;
        default: break;
    }
    if (rc != 0) return rc;
    return (int)cudaGetLastError();
}

extern "C" int ltq_matvec_slice(const uint8_t* data, int R, int K, int kbits, int frac, int h, int sub, const int* masks,
                                int n_masks, const float* lut, const float* gain_tab, const uint16_t* d_row,
                                const int8_t* e, long long ld_e, const float* x_rot, float* y, void* stream)
{
    if (!fmt_ok(R, K, kbits, frac, h, sub) || K % 256 || kbits > 6 || !masks || n_masks < 1 || n_masks > 3 || !lut ||
        (h > 0 && !gain_tab) || !d_row || !e || ld_e < K / 256 || !x_rot || !y || ((uintptr_t)data & 63) ||
        ((uintptr_t)x_rot & 15))
        return -1;
    DecodeArgs d{};
    d.p = pack_args(R, K, kbits, frac, h, sub);
    d.m0 = (unsigned)masks[0];
    d.m1 = n_masks > 1 ? (unsigned)masks[1] : 0u;
    d.m2 = n_masks > 2 ? (unsigned)masks[2] : 0u;
    d.nmask = n_masks;
    if (R == 0) return 0;
    const int nwarps = K / 256 < 32 ? K / 256 : 32;
    if (nwarps == 0) return -1;
    const unsigned grid = (unsigned)(R / 16);
    const cudaStream_t st = (cudaStream_t)stream;
    int rc = -1;
    switch (kbits) {
        case 2: rc = launch_matvec_kb<2>(frac, grid, 32 * nwarps, st, data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 3: rc = launch_matvec_kb<3>(frac, grid, 32 * nwarps, st, data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 4: rc = launch_matvec_kb<4>(frac, grid, 32 * nwarps, st, data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 5: rc = launch_matvec_kb<5>(frac, grid, 32 * nwarps, st, data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        case 6: rc = launch_matvec_kb<6>(frac, grid, 32 * nwarps, st, data, lut, gain_tab, d_row, e, ld_e, x_rot, y, d); break;
        default: break;
    }
    if (rc != 0) return rc;
    return (int)cudaGetLastError();
}
