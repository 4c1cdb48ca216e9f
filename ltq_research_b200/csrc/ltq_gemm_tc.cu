// Tensor-core GEMM for the quantizer's fp32-accurate products on B200 (sm_100a): tcgen05.mma with the accumulator in
// tensor memory, operands brought to shared memory by TMA.
//
//     C[M, N] = beta * C + alpha * A[M, Kd] B[N, Kd]^T      (A, B bf16 with K contiguous; fp32 accumulation and C)
//
// Used for the LDLQ inter-block update W_work[:, c1:] -= acat @ bcat_b (src/liqk_v2.py:972-979 in its six-product
// bf16 form: A = [e0 e0 e1 e0 e1 e2], B^T = the matching slots of U[c0:c1, c1:]) and the Cholesky panel / trailing
// products (src/liqk_v2.py:1078) of the fast mode, where the bf16 split makes every operand K-major.
//
// One CTA per 128 x 256 tile of C, 128 threads:
//   thread 0 (warp 0)  TMA producer: per 64-wide K chunk, A [128 x 64] and B [256 x 64] tiles into a ring of STAGES
//                      shared buffers (128-byte swizzle), completion counted in bytes on the stage's "full" mbarrier;
//   thread 32 (warp 1) MMA issuer: four tcgen05.mma (M 128, N 256, K 16 each) per chunk into one 128-lane x 256-column
//                      fp32 accumulator in tensor memory; tcgen05.commit frees the stage ("empty" mbarrier) once the
//                      MMAs have read it, and signals the accumulator after the last chunk;
//                      the other lanes of warps 0 and 1 wait at __syncwarp, so the two role threads issue alone;
//   all four warps     epilogue: warp w reads lanes 32 w .. 32 w + 31 (rows of the tile) with tcgen05.ld; for beta 0 / 1
//                      32 x 32 boxes go through swizzled shared buffers to a TMA store (beta 0) or a TMA reduce-add
//                      into C (beta 1), so C is never read by the SMs; any other beta reads and writes C row by row.
// gemm_bf16x3p_tn_kernel (below) is the same pipeline over compact three-part operands, batched over blockIdx.z;
// gemm_bf16x3p_tn_persist runs its beta 0 / 1 products of more tiles than SMs, one CTA per SM walking the tiles with a
// double-buffered accumulator so that epilogue and operand loads overlap the MMAs (bit-identical results).
// Every wait on an mbarrier is bounded: after GEMM_WAIT_LIMIT polls the thread records a timeout in *err (when given)
// and leaves its loop; the CTA still meets at its final barrier and frees its tensor memory.  No cluster, no multicast:
// every TMA load reads this GPU's own memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>
#include "ltq_b200.h"

namespace {

#ifndef LTQ_GEMM_BN
#define LTQ_GEMM_BN 256
#endif
#ifndef LTQ_GEMM_PERSIST
#define LTQ_GEMM_PERSIST 1  // beta 0 / 1 products of ltq_gemm_bf16x3p_tn on the persistent kernel
#endif
#ifndef LTQ_GEMM_STAGES
#define LTQ_GEMM_STAGES 2
#endif
constexpr int BM = 128, BN = LTQ_GEMM_BN, BK = 64, STAGES = LTQ_GEMM_STAGES;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB, a multiple of the 1024-byte swizzle atom
// two stages (97 KB of shared memory) let two CTAs share an SM, which measured faster than three stages at one CTA
constexpr int TMEM_COLS = BN;  // a power of two >= 32
constexpr uint32_t GEMM_WAIT_LIMIT = 1u << 26;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /* alignment */ + 256 /* barriers */;
static_assert(4 * 32 * ((BN < 128 ? BN : 128) + 4) * 4 <= STAGES * STAGE_BYTES, "epilogue staging exceeds the buffers");

struct GemmParams {
    float* C;
    long long ldc, cbs;  // row stride, batch stride (elements)
    int M, N, Kd;
    float alpha, beta;
    int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait for the phase with parity `parity`; false after `limit` polls (the timeout is recorded in *err)
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err, uint32_t limit = GEMM_WAIT_LIMIT)
{
    for (uint32_t i = 0; i < limit; i++)
        if (mbar_try_wait(b, parity)) return true;
    if (err) atomicExch(err, 1);
    return false;
}

// Self-test of the bounded wait: one thread waits on a fresh mbarrier that expects one arrival; with arrive = 1 the
// arrival is made first and the wait completes (*done = 1), with arrive = 0 nothing arrives and the wait gives up after
// `limit` polls, sets *err and returns (*done = 2).  No copy, no tensor memory: the timeout path runs without a fault.
__global__ void gemm_wait_selftest_kernel(int arrive, uint32_t limit, int* err, int* done)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        if (arrive) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(&bar)) : "memory");
        *done = mbar_wait(&bar, 0, err, limit) ? 1 : 2;
    }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// shared-memory matrix descriptor (tcgen05): K-major tile of rows x 64 bf16 with the 128-byte swizzle, as TMA writes it:
// 8-row atoms of 1024 bytes one after the other (stride byte offset 1024), the second 16-byte column chunk adjacent
// (leading byte offset 16), descriptor version 1, layout 2 (128-byte swizzle).  `addr` may step through the atom's
// row in 32-byte units (one K = 16 slice of bf16), the hardware applying the swizzle to the computed address.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t addr)
{
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both K-major
// (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Epilogue for beta = 0 or 1 without reading C: per warp, 32 rows x 32 columns at a time go from tensor memory (thread
// = row) to a 4 KB shared buffer in the 128-byte-swizzled layout of a {32 x 32} fp32 box (row r's 16-byte chunk k at
// chunk k ^ (r & 7): conflict-free 16-byte stores), then one lane has TMA store the box into C (beta 0) or add it to C
// in L2 (beta 1, cp.reduce.async.bulk.tensor .add: C + alpha acc in one rounding).  Two buffers per warp alternate;
// rows >= M and columns >= N of a box are clipped by the tensor map.  Deterministic: one CTA owns each element.
__device__ __forceinline__ void tma_store_box(const CUtensorMap* map, const void* src, int x, int y, int z, bool reduce)
{
    if (reduce)
        asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];\n" ::"l"(
                         map),
                     "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                     : "memory");
    else
        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];\n" ::"l"(map),
                     "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                     : "memory");
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}

__device__ __forceinline__ void epilogue_tma(const GemmParams& p, const CUtensorMap* tmC, bool reduce, uint64_t* accum,
                                             uint32_t tmem, uint8_t* smem, int m0, int n0, int warp, int lane)
{
    const bool ok = mbar_wait(accum, 0, p.err);
    __syncwarp();
    tc_fence_after();
    if (!ok) return;
    uint8_t* wbuf = smem + warp * 8192;
    const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);
    int nbox = 0;
    for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= p.N) break;  // warp-uniform
        float v[16], w[16];
        tmem_ld16(tl + c, v);
        tmem_ld16(tl + c + 16, w);
        uint8_t* buf = wbuf + (nbox & 1) * 4096;
        if (nbox >= 2) {  // the box stored from this buffer two boxes ago has been read out of shared memory
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
            __syncwarp();
        }
        uint8_t* row = buf + lane * 128;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            *reinterpret_cast<float4*>(row + ((q ^ (lane & 7)) << 4)) =
                make_float4(p.alpha * v[4 * q], p.alpha * v[4 * q + 1], p.alpha * v[4 * q + 2], p.alpha * v[4 * q + 3]);
            *reinterpret_cast<float4*>(row + (((q + 4) ^ (lane & 7)) << 4)) =
                make_float4(p.alpha * w[4 * q], p.alpha * w[4 * q + 1], p.alpha * w[4 * q + 2], p.alpha * w[4 * q + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // the writes, visible to the TMA engine
        __syncwarp();
        if (lane == 0) tma_store_box(tmC, buf, n0 + c, m0 + 32 * warp, blockIdx.z, reduce);
        nbox++;
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    __syncwarp();
}

// Epilogue, in halves of 128 columns: each warp moves its 32 rows x 16 columns at a time from tensor memory (thread =
// row) into a row-major shared tile (the pipeline's buffers are free once the accumulator is complete), then writes C
// row by row, a whole 512-byte row segment per warp instruction (coalesced read-modify-write), C = beta C + alpha acc.
__device__ __forceinline__ void epilogue(const GemmParams& p, uint64_t* accum, uint32_t tmem, uint8_t* smem, int m0,
                                         int n0, int warp, int lane)
{
    const bool ok = mbar_wait(accum, 0, p.err);
    __syncwarp();
    tc_fence_after();
    if (!ok) return;
    constexpr int HALF = BN < 128 ? BN : 128, LDS = HALF + 4;
    float* st = reinterpret_cast<float*>(smem) + warp * 32 * LDS;
    const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);
    for (int h = 0; h < BN; h += HALF) {
        if (n0 + h >= p.N) break;  // warp-uniform
        for (int c = 0; c < HALF; c += 16) {
            float v[16];
            tmem_ld16(tl + h + c, v);
#pragma unroll
            for (int q = 0; q < 4; q++)
                *reinterpret_cast<float4*>(st + lane * LDS + c + 4 * q) =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        __syncwarp();
        const int col = n0 + h + 4 * lane;
        for (int r = 0; r < 32; r++) {
            const int row = m0 + 32 * warp + r;
            if (row >= p.M) break;
            if (col < p.N) {
                const float4 a = *reinterpret_cast<const float4*>(st + r * LDS + 4 * lane);
                float* cp = p.C + (long long)blockIdx.z * p.cbs + (long long)row * p.ldc + col;
                float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
                if (p.beta != 0.f) {
                    const float4 old = *reinterpret_cast<const float4*>(cp);
                    o = make_float4(p.beta * old.x, p.beta * old.y, p.beta * old.z, p.beta * old.w);
                }
                o.x = __fmaf_rn(p.alpha, a.x, o.x);
                o.y = __fmaf_rn(p.alpha, a.y, o.y);
                o.z = __fmaf_rn(p.alpha, a.z, o.z);
                o.w = __fmaf_rn(p.alpha, a.w, o.w);
                *reinterpret_cast<float4*>(cp) = o;
            }
        }
        __syncwarp();
    }
}

__global__ void __launch_bounds__(128, 1) gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA,
                                                              const __grid_constant__ CUtensorMap tmB,
                                                              const __grid_constant__ CUtensorMap tmC,
                                                              const GemmParams p, const int cmode)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int nk = p.Kd / BK;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmB) : "memory");
        if (cmode) asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmC) : "memory");
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {  // the whole warp allocates the accumulator's columns (the address lands in shared memory)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // roles: lane 0 of warp 0 feeds the pipeline, lane 0 of warp 1 issues the MMAs; their warps' other lanes wait at
    // the warp's own barrier (not on an mbarrier: a spinning sibling path would be serialised with the role's path and
    // delay it), then every warp runs the epilogue
    if (warp == 0) {
        if (lane == 0) {  // TMA producer
        int issued = 0;
        for (int k = 0; k < nk; k++) {
            const int s = k % STAGES;
            if (k >= STAGES && !mbar_wait(&empty[s], ((k / STAGES) - 1) & 1, p.err)) break;
            mbar_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(smem + s * STAGE_BYTES, &tmA, k * BK, m0, &full[s]);
            tma_load_2d(smem + s * STAGE_BYTES + A_BYTES, &tmB, k * BK, n0, &full[s]);
            issued = k + 1;
        }
        // every copy this thread started has landed before the CTA can leave (a completed phase stays visible to
        // its parity until the barrier completes the next one, which needs a new arrive from this thread)
        for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; k++)
            mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
        for (int k = 0; k < nk; k++) {
            const int s = k % STAGES;
            if (!mbar_wait(&full[s], (k / STAGES) & 1, p.err)) break;
            tc_fence_after();
            const uint32_t a = smem_u32(smem + s * STAGE_BYTES), b = a + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++)
                umma_bf16(tmem, sw128_kmajor_desc(a + 32 * kk), sw128_kmajor_desc(b + 32 * kk), (k | kk) != 0);
            umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        umma_commit(accum);  // arrives when every MMA issued above has completed
        }
        __syncwarp();
    }

    if (cmode == 0) epilogue(p, accum, tmem, smem, m0, n0, warp, lane);
    else epilogue_tma(p, &tmC, cmode == 2, accum, tmem, smem, m0, n0, warp, lane);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// Products of split fp32 operands from compact part operands: A3 = [a0 a1 a2] [M, 3 Kp] and B3 = [b0 b1 b2] [N, 3 Kp]
// (bf16, K contiguous; x = x0 + x1 + x2 the three-way split of an fp32 matrix), batched over blockIdx.z:
//     C = beta C + alpha sum_{p + q < nq} a_p b_q^T
// nq = 3: the six products a0 b0 + a1 b0 + a2 b0 + a0 b1 + a1 b1 + a0 b2 (an fp32-accurate product);
// nq = 2: the three products a0 b0 + a1 b0 + a0 b1 (a product whose own size makes fp32 rounding of its terms moot).
// Per 64-wide chunk j of Kp: the A parts of the chunk stay in one of two A buffers (3 x 16 KB) while the B parts stream
// through three 32 KB stages (stage q holds b_q): b0 meets a0 .. a_{nq-1}, b1 meets a0 .. a_{nq-2}, ... — each A part
// of a chunk loaded once for every B part it meets, half the operand bytes of the concatenated six-slot form.
constexpr int A3_BYTES = 3 * A_BYTES;
constexpr int SMEM6_BYTES = 2 * A3_BYTES + 3 * B_BYTES + 1024 + 256;
static_assert(4 * 32 * ((BN < 128 ? BN : 128) + 4) * 4 <= 2 * A3_BYTES + 3 * B_BYTES, "epilogue staging");

__global__ void __launch_bounds__(128, 1) gemm_bf16x3p_tn_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                 const __grid_constant__ CUtensorMap tmB,
                                                                 const __grid_constant__ CUtensorMap tmC,
                                                                 const GemmParams p, const int cmode, const int Kp,
                                                                 const int nq)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sa = smem;                   // 2 A buffers of nq parts
    uint8_t* sb = smem + 2 * A3_BYTES;    // B stages (stage q = part q)
    uint64_t* afull = reinterpret_cast<uint64_t*>(sb + 3 * B_BYTES);
    uint64_t* aempty = afull + 2;
    uint64_t* bfull = aempty + 2;
    uint64_t* bempty = bfull + 3;
    uint64_t* accum = bempty + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN, z = blockIdx.z;
    const int nk = Kp / BK;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmB) : "memory");
        if (cmode) asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmC) : "memory");
        for (int i = 0; i < 2; i++) {
            mbar_init(&afull[i], 1);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < 3; i++) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // roles as in gemm_bf16_tn_kernel: lane 0 of warp 0 loads, lane 0 of warp 1 issues the MMAs, their siblings wait at
    // __syncwarp, then every warp runs the epilogue
    if (warp == 0) {
        if (lane == 0) {  // TMA producer: per chunk j, the A parts, then b0 .. b_{nq-1}
            int ja = 0, jb = 0;  // chunks whose A / B loads were all issued
            for (int j = 0; j < nk; j++) {
                const int a = j & 1;
                if (j >= 2 && !mbar_wait(&aempty[a], ((j >> 1) - 1) & 1, p.err)) break;
                mbar_expect_tx(&afull[a], nq * A_BYTES);
                for (int pt = 0; pt < nq; pt++)
                    tma_load_3d(sa + a * A3_BYTES + pt * A_BYTES, &tmA, pt * Kp + j * BK, m0, z, &afull[a]);
                ja = j + 1;
                bool ok = true;
                for (int q = 0; q < nq; q++) {
                    if (j >= 1 && !mbar_wait(&bempty[q], (j - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&bfull[q], B_BYTES);
                    tma_load_3d(sb + q * B_BYTES, &tmB, q * Kp + j * BK, n0, z, &bfull[q]);
                }
                if (!ok) break;
                jb = j + 1;
            }
            // every copy started has landed before the CTA can leave
            for (int j = ja > 2 ? ja - 2 : 0; j < ja; j++) mbar_wait(&afull[j & 1], (j >> 1) & 1, p.err);
            if (jb > 0)
                for (int q = 0; q < nq; q++) mbar_wait(&bfull[q], (jb - 1) & 1, p.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            bool ok = true, first = true;
            for (int j = 0; j < nk && ok; j++) {
                const int a = j & 1;
                if (!mbar_wait(&afull[a], (j >> 1) & 1, p.err)) break;
                const uint32_t abase = smem_u32(sa + a * A3_BYTES);
                for (int q = 0; q < nq; q++) {
                    if (!mbar_wait(&bfull[q], j & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bq = smem_u32(sb + q * B_BYTES);
                    for (int pt = 0; pt < nq - q; pt++) {
                        const uint32_t ap = abase + pt * A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            umma_bf16(tmem, sw128_kmajor_desc(ap + 32 * kk), sw128_kmajor_desc(bq + 32 * kk),
                                      first ? 0u : 1u);
                            first = false;
                        }
                    }
                    umma_commit(&bempty[q]);
                }
                if (ok) umma_commit(&aempty[a]);
            }
            umma_commit(accum);
        }
        __syncwarp();
    }
    if (cmode == 0) epilogue(p, accum, tmem, smem, m0, n0, warp, lane);
    else epilogue_tma(p, &tmC, cmode == 2, accum, tmem, smem, m0, n0, warp, lane);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
    PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
    if (!f) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        fn.store(f, std::memory_order_release);
    }
    return f;
}

// Persistent form of gemm_bf16x3p_tn_kernel for beta 0 / 1 (TMA store / reduce-add epilogue): one CTA per SM walks
// the tiles (tile t: batch z, row block, column block; t += gridDim.x) with warp-specialised roles,
//   warp 0 lane 0   TMA producer, the A / B rings of the one-tile kernel continued across tiles;
//   warp 1 lane 0   MMA issuer into one of two 256-column accumulators in tensor memory (512 columns), tile i into
//                   accumulator i & 1, once the epilogue has released it (accempty), then accfull;
//   warps 2 .. 5    epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (its lane quarter), stages 32 x 32
//                   boxes in its own 8 KB of shared memory and stores / adds them with TMA, then releases the
//                   accumulator —
// so the epilogue of tile i and the operand loads of tile i + 1 overlap the MMAs instead of following them.  Every wait
// is bounded (GEMM_WAIT_LIMIT polls, then *err = 1 and the role stops); the CTA still meets at its last barrier.
constexpr int PERSIST_STAGE = 4 * 8192;  // epilogue staging: 4 warps x two 4 KB boxes
constexpr int SMEM6P_BYTES = 2 * A3_BYTES + 3 * B_BYTES + PERSIST_STAGE + 1024 + 256;

__global__ void __launch_bounds__(192, 1) gemm_bf16x3p_tn_persist(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ CUtensorMap tmB,
                                                                  const __grid_constant__ CUtensorMap tmC,
                                                                  const GemmParams p, const int reduce, const int Kp,
                                                                  const int nq, const int mt, const int ntl,
                                                                  const int ntiles)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sa = smem;                   // 2 A buffers of nq parts
    uint8_t* sb = smem + 2 * A3_BYTES;    // B stages (stage q = part q)
    uint8_t* sst = sb + 3 * B_BYTES;      // epilogue staging
    uint64_t* afull = reinterpret_cast<uint64_t*>(sst + PERSIST_STAGE);
    uint64_t* aempty = afull + 2;
    uint64_t* bfull = aempty + 2;
    uint64_t* bempty = bfull + 3;
    uint64_t* accfull = bempty + 3;
    uint64_t* accempty = accfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = Kp / BK;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmB) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmC) : "memory");
        for (int i = 0; i < 2; i++) {
            mbar_init(&afull[i], 1);
            mbar_init(&aempty[i], 1);
            mbar_init(&accfull[i], 1);
            mbar_init(&accempty[i], 4);  // one arrival per epilogue warp
        }
        for (int i = 0; i < 3; i++) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto tile_of = [&](int t, int& m0, int& n0, int& z) {
        z = t / (mt * ntl);
        const int r = t - z * mt * ntl;
        n0 = (r / mt) * BN;  // consecutive tiles share a column block (its B operand stays in L2)
        m0 = (r % mt) * BM;
    };
    if (warp == 0) {
        if (lane == 0) {  // TMA producer; g counts chunks over all of this CTA's tiles
            int g = 0, ga = 0, lastb[3] = {-1, -1, -1};
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                int m0, n0, z;
                tile_of(t, m0, n0, z);
                for (int j = 0; j < nk && ok; j++, g++) {
                    const int a = g & 1;
                    if (g >= 2 && !mbar_wait(&aempty[a], ((g >> 1) - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&afull[a], nq * A_BYTES);
                    for (int pt = 0; pt < nq; pt++)
                        tma_load_3d(sa + a * A3_BYTES + pt * A_BYTES, &tmA, pt * Kp + j * BK, m0, z, &afull[a]);
                    ga = g + 1;
#pragma unroll
                    for (int q = 0; q < 3; q++) {
                        if (q >= nq) break;
                        if (g >= 1 && !mbar_wait(&bempty[q], (g - 1) & 1, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&bfull[q], B_BYTES);
                        tma_load_3d(sb + q * B_BYTES, &tmB, q * Kp + j * BK, n0, z, &bfull[q]);
                        lastb[q] = g;
                    }
                }
            }
            // every copy started has landed before the CTA can leave
            for (int h = ga > 2 ? ga - 2 : 0; h < ga; h++) mbar_wait(&afull[h & 1], (h >> 1) & 1, p.err);
#pragma unroll
            for (int q = 0; q < 3; q++)
                if (lastb[q] >= 0) mbar_wait(&bfull[q], lastb[q] & 1, p.err);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int g = 0, i = 0, last = -1;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, i++) {
                const int acc = i & 1;
                if (i >= 2 && !mbar_wait(&accempty[acc], ((i >> 1) - 1) & 1, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * BN);
                bool first = true;
                for (int j = 0; j < nk && ok; j++, g++) {
                    const int a = g & 1;
                    if (!mbar_wait(&afull[a], (g >> 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t abase = smem_u32(sa + a * A3_BYTES);
                    for (int q = 0; q < nq; q++) {
                        if (!mbar_wait(&bfull[q], g & 1, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t bq = smem_u32(sb + q * B_BYTES);
                        for (int pt = 0; pt < nq - q; pt++) {
                            const uint32_t ap = abase + pt * A_BYTES;
#pragma unroll
                            for (int kk = 0; kk < BK / 16; kk++) {
                                umma_bf16(d, sw128_kmajor_desc(ap + 32 * kk), sw128_kmajor_desc(bq + 32 * kk),
                                          first ? 0u : 1u);
                                first = false;
                            }
                        }
                        umma_commit(&bempty[q]);
                    }
                    if (ok) umma_commit(&aempty[a]);
                }
                umma_commit(&accfull[acc]);  // arrives when every MMA issued so far has completed
                last = i;
            }
            // no MMA may still write tensor memory when the CTA frees it
            if (last >= 0) mbar_wait(&accfull[last & 1], (last >> 1) & 1, p.err);
        }
        __syncwarp();
    } else {  // epilogue warps: lane quarter qr of tensor memory, rows m0 + 32 qr .. + 31
        const int qr = warp & 3;
        uint8_t* wbuf = sst + (warp - 2) * 8192;
        int nbox = 0, i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
            int m0, n0, z;
            tile_of(t, m0, n0, z);
            const int acc = i & 1;
            const bool ok = mbar_wait(&accfull[acc], (i >> 1) & 1, p.err);
            __syncwarp();
            tc_fence_after();
            if (!ok) break;
            const uint32_t tl = tmem + ((uint32_t)(32 * qr) << 16) + (uint32_t)(acc * BN);
            for (int c = 0; c < BN; c += 32) {
                if (n0 + c >= p.N) break;  // warp-uniform
                float v[16], w[16];
                tmem_ld16(tl + c, v);
                tmem_ld16(tl + c + 16, w);
                uint8_t* buf = wbuf + (nbox & 1) * 4096;
                if (nbox >= 2) {  // the box stored from this buffer two boxes ago has been read out of shared memory
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
                    __syncwarp();
                }
                uint8_t* row = buf + lane * 128;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    *reinterpret_cast<float4*>(row + ((q ^ (lane & 7)) << 4)) = make_float4(
                        p.alpha * v[4 * q], p.alpha * v[4 * q + 1], p.alpha * v[4 * q + 2], p.alpha * v[4 * q + 3]);
                    *reinterpret_cast<float4*>(row + (((q + 4) ^ (lane & 7)) << 4)) = make_float4(
                        p.alpha * w[4 * q], p.alpha * w[4 * q + 1], p.alpha * w[4 * q + 2], p.alpha * w[4 * q + 3]);
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) tma_store_box(&tmC, buf, n0 + c, m0 + 32 * qr, z, reduce != 0);
                nbox++;
            }
            // this warp's reads of the accumulator are complete (tcgen05.wait::ld): hand it back to the MMA issuer
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(&accempty[acc])) : "memory");
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512) : "memory");
    }
}
static_assert(2 * BN == 512, "two accumulators of BN columns fill the 512 columns of tensor memory");
static_assert(SMEM6P_BYTES <= 232448, "shared memory of one CTA");
// 3-D tensor map of the fp32 output C [batch][rows, cols] (row stride ld, batch stride bs elements) for the epilogue's
// {32 x 32 x 1} boxes, 128-byte swizzle
bool make_map_c(CUtensorMap* m, const float* base, int rows, int cols, long long ld, int batch, long long bs)
{
    auto f = encode_fn();
    if (!f) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(batch > 1 ? bs : ld * rows) * 4};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D tensor map of a bf16 operand [batch][rows, cols] (row stride ld, batch stride bs elements), box
// [1][box_rows][64], 128-byte swizzle; out-of-range rows and columns read as zero
bool make_map3(CUtensorMap* m, const void* base, int rows, int cols, long long ld, int batch, long long bs,
               int box_rows)
{
    auto f = encode_fn();
    if (!f) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(batch > 1 ? bs : ld * rows) * 2};
    cuuint32_t box[3] = {BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// epilogue mode: 1 TMA store (beta 0), 2 TMA reduce-add (beta 1), 0 read-modify-write (any other beta)
int c_mode(float beta) { return beta == 0.f ? 1 : (beta == 1.f ? 2 : 0); }

// 2-D tensor map of a row-major bf16 matrix [rows, cols] (row stride ld elements), box [box_rows, 64] with the
// 128-byte swizzle; out-of-range rows and columns read as zero
bool make_map(CUtensorMap* m, const void* base, int rows, int cols, long long ld, int box_rows)
{
    auto f = encode_fn();
    if (!f) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int ltq_gemm_wait_selftest(int arrive, unsigned int limit, int* err, int* done, void* stream)
{
    if (!err || !done || limit == 0 || limit > GEMM_WAIT_LIMIT) return -1;
    gemm_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(arrive, limit, err, done);
    return (int)cudaGetLastError();
}

extern "C" int ltq_gemm_bf16_tn(const uint16_t* A, long long lda, const uint16_t* B, long long ldb, float* C,
                                long long ldc, int M, int N, int Kd, float alpha, float beta, int* err, void* stream)
{
    if (M < 0 || N < 0 || Kd < 0 || N % 16 || Kd % BK || !A || !B || !C || lda < Kd || ldb < Kd || ldc < N ||
        (lda % 8) || (ldb % 8) || (ldc % 4) || ((uintptr_t)A & 15) || ((uintptr_t)B & 15) || ((uintptr_t)C & 15))
        return -1;
    if (M == 0 || N == 0) return 0;
    if (Kd == 0) return -1;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, M, Kd, lda, BM) || !make_map(&tb, B, N, Kd, ldb, BN)) return -1;
    static std::atomic<int> attr_set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(gemm_bf16_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return -1;
        attr_set[dev].store(1, std::memory_order_release);
    }
    const int cm = c_mode(beta);
    CUtensorMap tc{};
    if (cm && !make_map_c(&tc, C, M, N, ldc, 1, 0)) return -1;
    GemmParams p{C, ldc, 0, M, N, Kd, alpha, beta, err};
    dim3 grid((M + BM - 1) / BM, (N + BN - 1) / BN);
    gemm_bf16_tn_kernel<<<grid, 128, SMEM_BYTES, (cudaStream_t)stream>>>(ta, tb, tc, p, cm);
    return (int)cudaGetLastError();
}

extern "C" int ltq_gemm_bf16x3p_tn(const uint16_t* A3, long long lda, long long abs_, const uint16_t* B3,
                                   long long ldb, long long bbs, float* C, long long ldc, long long cbs, int M, int N,
                                   int Kp, int nq, int batch, float alpha, float beta, int* err, void* stream)
{
    if (M < 0 || N < 0 || Kp <= 0 || N % 16 || Kp % BK || (nq != 2 && nq != 3) || batch < 1 || batch > 65535 || !A3 ||
        !B3 || !C || lda < 1LL * nq * Kp || ldb < 1LL * nq * Kp || ldc < N || (lda % 8) || (ldb % 8) || (ldc % 4) ||
        ((uintptr_t)A3 & 15) || ((uintptr_t)B3 & 15) || ((uintptr_t)C & 15) ||
        (batch > 1 && (abs_ % 8 || bbs % 8 || cbs % 4 || abs_ < lda * M || bbs < ldb * N || cbs < ldc * M)))
        return -1;
    if (M == 0 || N == 0) return 0;
    CUtensorMap ta, tb;
    if (!make_map3(&ta, A3, M, nq * Kp, lda, batch, abs_, BM) || !make_map3(&tb, B3, N, nq * Kp, ldb, batch, bbs, BN))
        return -1;
    static std::atomic<int> attr_set[64];
    static int sm_count[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(gemm_bf16x3p_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM6_BYTES) !=
                cudaSuccess ||
            cudaFuncSetAttribute(gemm_bf16x3p_tn_persist, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SMEM6P_BYTES) != cudaSuccess ||
            cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return -1;
        attr_set[dev].store(1, std::memory_order_release);
    }
    const int cm = c_mode(beta);
    CUtensorMap tc{};
    if (cm && !make_map_c(&tc, C, M, N, ldc, batch, cbs)) return -1;
    GemmParams p{C, ldc, cbs, M, N, Kp, alpha, beta, err};
    const int mt = (M + BM - 1) / BM, ntl = (N + BN - 1) / BN;
    const long long ntiles = 1LL * mt * ntl * batch;
    // more tiles than SMs: the persistent kernel (one wave is faster on the one-tile kernel, which starts lighter)
    if (cm && LTQ_GEMM_PERSIST && ntiles > sm_count[dev] && ntiles < (1LL << 31)) {
        gemm_bf16x3p_tn_persist<<<sm_count[dev], 192, SMEM6P_BYTES, (cudaStream_t)stream>>>(ta, tb, tc, p, cm == 2, Kp, nq, mt,
                                                                                   ntl, (int)ntiles);
    } else {
        dim3 grid(mt, ntl, batch);
        gemm_bf16x3p_tn_kernel<<<grid, 128, SMEM6_BYTES, (cudaStream_t)stream>>>(ta, tb, tc, p, cm, Kp, nq);
    }
    return (int)cudaGetLastError();
}

extern "C" int ltq_gemm_bf16x6_tn(const uint16_t* A3, long long lda, const uint16_t* B3, long long ldb, float* C,
                                  long long ldc, int M, int N, int Kp, float alpha, float beta, int* err, void* stream)
{
    return ltq_gemm_bf16x3p_tn(A3, lda, 0, B3, ldb, 0, C, ldc, 0, M, N, Kp, 3, 1, alpha, beta, err, stream);
}
