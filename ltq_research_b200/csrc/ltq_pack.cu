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
// ltq_pack_slice_kernel / ltq_decode_slice_kernel: one warp per tile.  Lane L owns row L / 2, columns 8 (L & 1) .. + 7
// (one 16-byte load of idx, one 8-byte load of gi); a field word is assembled from the owning lanes' bit fragments with
// warp shuffles.  Both are HBM-bound (3 bytes read per weight for packing, tile_bytes / 256 written).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "ltq_b200.h"

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

__global__ void __launch_bounds__(256) ltq_pack_slice_kernel(const int16_t* __restrict__ idx,
                                                             const uint8_t* __restrict__ gi, long long ld,
                                                             uint8_t* __restrict__ out, const PackArgs a)
{
    const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.T) return;
    const int lane = threadIdx.x & 31, r = lane >> 1, hf = lane & 1;
    const long long rg = t / a.tiles_per_row, kb = t % a.tiles_per_row;
    const long long base = (rg * 16 + r) * ld + kb * 16 + 8 * hf;
    const uint4 iv = *reinterpret_cast<const uint4*>(idx + base);
    const uint2 gv = *reinterpret_cast<const uint2*>(gi + base);
    const int16_t* ix = reinterpret_cast<const int16_t*>(&iv);
    const uint8_t* gx = reinterpret_cast<const uint8_t*>(&gv);
    const int U = 1 << (a.kbits - 1);
    uint32_t cb = 0, lsb = 0, pl[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int v = (int)(uint16_t)ix[j];
        const int lab = v / U, u = v % U;
        cb |= (uint32_t)(lab & 1) << j;
        lsb |= (uint32_t)(u & 1) << j;
#pragma unroll
        for (int p = 1; p < 7; p++)
            if (p < a.kbits - 1) pl[p - 1] |= (uint32_t)((u >> p) & 1) << j;
    }
    // codes and planes: lane l holds 8 bits at 8 l
    uint16_t* reg0 = reinterpret_cast<uint16_t*>(out + a.off[0]) + t * a.nw[0];
    const uint32_t cw = gather_word(cb, 8, lane);
    if (lane < 16) reg0[lane] = (uint16_t)cw;
    uint16_t* reg1 = reinterpret_cast<uint16_t*>(out + a.off[1]) + t * a.nw[1];
    for (int p = 1; p < a.kbits - 1; p++) {
        uint32_t v = 0;
#pragma unroll
        for (int q = 0; q < 6; q++)
            if (q == p - 1) v = pl[q];
        const uint32_t pw = gather_word(v, 8, lane);
        if (lane < 16) reg1[(p - 1) * 16 + lane] = (uint16_t)pw;
    }
    // lsb: all 8 bits (frac 0), the 4 even positions (D2), the first 3 of each of the 2 quads (D4)
    uint32_t lv;
    int nb;
    if (a.frac == 0) {
        lv = lsb; nb = 8;
    } else if (a.frac == 1) {
        lv = (lsb & 1) | ((lsb >> 1) & 2) | ((lsb >> 2) & 4) | ((lsb >> 3) & 8); nb = 4;
    } else {
        lv = (lsb & 7) | (((lsb >> 4) & 7) << 3); nb = 6;
    }
    uint16_t* reg2 = reinterpret_cast<uint16_t*>(out + a.off[2]) + t * a.nw[2];
    const uint32_t lw = gather_word(lv, nb, lane);
    if (lane < a.nw[2]) reg2[lane] = (uint16_t)lw;
    // gains: the index at the first position of sub-block k (row k sub / 16, column 0, i.e. lane 2 (k sub / 16),
    // element 0) moves to lane k, which then holds h bits at h k
    if (a.h > 0) {
        const int nsb = 256 / a.sub;
        const uint32_t g0 = gx[0];
        const uint32_t gk = __shfl_sync(FULL, g0, (2 * ((lane * a.sub) >> 4)) & 31);
        const uint32_t v = lane < nsb ? (gk & ((1u << a.h) - 1u)) : 0u;
        uint16_t* reg3 = reinterpret_cast<uint16_t*>(out + a.off[3]) + t * a.nw[3];
        const uint32_t gw = gather_word(v, a.h, lane);
        if (lane < a.nw[3]) reg3[lane] = (uint16_t)gw;
    }
}

struct DecodeArgs {
    PackArgs p;
    unsigned m0, m1, m2;
    int nmask;
};

__device__ __forceinline__ int bit_of(const uint32_t (&w)[8], int b) { return (w[b >> 5] >> (b & 31)) & 1; }

__global__ void __launch_bounds__(256) ltq_decode_slice_kernel(const uint8_t* __restrict__ data,
                                                               const float* __restrict__ lut,
                                                               const float* __restrict__ gain_tab,
                                                               float* __restrict__ out, long long ld_out,
                                                               const float* __restrict__ ref, long long ld_ref,
                                                               unsigned long long* __restrict__ mismatches,
                                                               const DecodeArgs d)
{
    const PackArgs& a = d.p;
    const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.T) return;
    const int lane = threadIdx.x & 31, r = lane >> 1, hf = lane & 1;
    const long long rg = t / a.tiles_per_row, kb = t % a.tiles_per_row;
    const int U = 1 << (a.kbits - 1);
    // the whole code-bit string of the tile (256 bits) in every lane: states wrap around the tile (tail-biting)
    uint32_t cw[8];
    {
        const uint4* c4 = reinterpret_cast<const uint4*>(data + a.off[0] + t * 32);
        const uint4 x0 = c4[0], x1 = c4[1];
        cw[0] = x0.x; cw[1] = x0.y; cw[2] = x0.z; cw[3] = x0.w; cw[4] = x1.x; cw[5] = x1.y; cw[6] = x1.z; cw[7] = x1.w;
    }
    const uint16_t* pl = reinterpret_cast<const uint16_t*>(data + a.off[1]) + t * a.nw[1];
    const uint16_t* lw = reinterpret_cast<const uint16_t*>(data + a.off[2]) + t * a.nw[2];
    const uint16_t* gw = reinterpret_cast<const uint16_t*>(data + a.off[3]) + t * a.nw[3];
    unsigned bad = 0;
    float* orow = out ? out + (rg * 16 + r) * ld_out + kb * 16 + 8 * hf : nullptr;
    const float* rrow = ref ? ref + (rg * 16 + r) * ld_ref + kb * 16 + 8 * hf : nullptr;
#pragma unroll 2
    for (int j = 0; j < 8; j++) {
        const int pos = 16 * r + 8 * hf + j;
        unsigned s = 0;
#pragma unroll
        for (int q = 0; q < 10; q++) s |= (unsigned)bit_of(cw, (pos - q) & 255) << q;
        const unsigned v = s >> 1;
        int lab = (int)(s & 1) | ((__popc(v & d.m0) & 1) << 1);
        if (d.nmask > 1) lab |= (__popc(v & d.m1) & 1) << 2;
        if (d.nmask > 2) lab |= (__popc(v & d.m2) & 1) << 3;
        int u;
        if (a.frac == 0) {
            u = (lw[pos >> 4] >> (pos & 15)) & 1;
        } else if (a.frac == 1) {
            const int b = pos >> 1;
            u = (lw[b >> 4] >> (b & 15)) & 1;
        } else {
            const int q4 = pos >> 2, i = pos & 3;
            if (i < 3) {
                const int b = 3 * q4 + i;
                u = (lw[b >> 4] >> (b & 15)) & 1;
            } else {
                u = 0;
                for (int k = 0; k < 3; k++) {
                    const int b = 3 * q4 + k;
                    u ^= (lw[b >> 4] >> (b & 15)) & 1;
                }
            }
        }
        for (int p = 1; p < a.kbits - 1; p++) u |= ((pl[(p - 1) * 16 + r] >> (pos & 15)) & 1) << p;
        int g = 0;
        if (a.h > 0) {
            const int k = pos / a.sub;
            for (int i = 0; i < a.h; i++) {
                const int b = k * a.h + i;
                g |= ((gw[b >> 4] >> (b & 15)) & 1) << i;
            }
        }
        const float val = __fmul_rn(a.h > 0 ? gain_tab[g] : 1.0f, lut[lab * U + u]);
        if (orow) orow[j] = val;
        if (rrow && val != rrow[j]) bad++;
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
    cudaMemsetAsync(out, 0, (size_t)slice_layout(a.T, kbits, frac, h, sub).total, (cudaStream_t)stream);
    ltq_pack_slice_kernel<<<(unsigned)((a.T + 7) / 8), 256, 0, (cudaStream_t)stream>>>(idx, gi, ld, out, a);
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
    if (d.p.T == 0) return 0;
    ltq_decode_slice_kernel<<<(unsigned)((d.p.T + 7) / 8), 256, 0, (cudaStream_t)stream>>>(data, lut, gain_tab, out,
                                                                                          ld_out, ref, ld_ref,
                                                                                          mismatches, d);
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
