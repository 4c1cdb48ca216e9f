// Launch helpers for the Viterbi kernel instantiations (one translation unit per label-mask set).
#pragma once
#include <atomic>
#include "ldlq_block_kernel.cuh"
#include "tcq_viterbi_kernel.cuh"

namespace ltqb {

// Raise the kernel's dynamic shared-memory limit to the device maximum once per (kernel, device).  The limit is
// always set to the same value, so concurrent callers on other host threads cannot lower it under a launch.
// `done` is the caller's per-kernel flag array (one static array per kernel instantiation).
template <class K>
inline int ensure_smem(K kernel, int smem, std::atomic<int>* done)
{
    if (smem <= 48 * 1024) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (done[dev].load(std::memory_order_acquire)) return 0;
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return -1;
    const int want = optin - (int)fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want) != cudaSuccess) return -1;
    done[dev].store(1, std::memory_order_release);
    return smem <= want ? 0 : -1;
}

template <class MP, int MD, bool SUB2 = false>
inline int launch_one(const VitParams& p, int smem, cudaStream_t st)
{
    auto k = vit_fwd_kernel<MP, MD, SUB2>;
    static std::atomic<int> done[64];
    if (ensure_smem(k, smem, done) != 0) return -1;
    k<<<p.N, 32 * p.G, smem, st>>>(p);
    return 0;
}

// sub-blocks that are not a multiple of 4 steps (no format uses them) run the SUB2 variant, plain and D2 only
template <class MP>
inline int launch_md_sub2(const VitParams& p, int md, int smem, cudaStream_t st)
{
    switch (md) {
        case 0: return launch_one<MP, 0, true>(p, smem, st);
        case 1: return launch_one<MP, 1, true>(p, smem, st);
        default: return -1;
    }
}

template <class MP>
inline int launch_md(const VitParams& p, int md, int smem, cudaStream_t st)
{
    switch (md) {
        case 0: return launch_one<MP, 0>(p, smem, st);
        case 1: return launch_one<MP, 1>(p, smem, st);
        case 2: return launch_one<MP, 2>(p, smem, st);
        case 3: return launch_one<MP, 3>(p, smem, st);
        default: return -1;
    }
}

// fused LDLQ block (one CTA of 32 G threads per 16-row tile group)
template <class MP, int MD>
inline int launch_ldlq_one(const LdlqParams& q, int smem, int grid, cudaStream_t st)
{
    auto k = ldlq_block_kernel<MP, MD>;
    static std::atomic<int> done[64];
    if (ensure_smem(k, smem, done) != 0) return -1;
    k<<<grid, 32 * q.p2.G, smem, st>>>(q);
    return 0;
}

template <class MP>
inline int launch_ldlq_md(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st)
{
    switch (md) {
        case 0: return launch_ldlq_one<MP, 0>(q, smem, grid, st);
        case 1: return launch_ldlq_one<MP, 1>(q, smem, grid, st);
        case 2: return launch_ldlq_one<MP, 2>(q, smem, grid, st);
        case 3: return launch_ldlq_one<MP, 3>(q, smem, grid, st);
        default: return -1;
    }
}

// label-mask sets with compiled-in masks (every set used by the reference's format tables; primary mask 359)
int launch_ct_m359(const VitParams& p, int md, int smem, cudaStream_t st);          // 4 subsets
int launch_ct_m359_241(const VitParams& p, int md, int smem, cudaStream_t st);      // 8
int launch_ct_m359_462(const VitParams& p, int md, int smem, cudaStream_t st);      // 8
int launch_ct_m359_146(const VitParams& p, int md, int smem, cudaStream_t st);      // 8
int launch_ct_m359_58_299(const VitParams& p, int md, int smem, cudaStream_t st);   // 16
int launch_ct_m359_211_397(const VitParams& p, int md, int smem, cudaStream_t st);  // 16
int launch_ct_m359_40_475(const VitParams& p, int md, int smem, cudaStream_t st);   // 16
int launch_rt(const VitParams& p, int md, int smem, cudaStream_t st);               // any masks, nl 4 / 8 / 16
int launch_rt_sub2(const VitParams& p, int md, int smem, cudaStream_t st);          // any masks, sub = 2 mod 4
int launch_tb(const VitParams& p, int md, cudaStream_t st);                          // traceback + reconstruction
int run_pass_s256(VitParams p, cudaStream_t st);                                      // the 256-state trellis
// fused LDLQ block, per label-mask set (same sets as the forward kernel)
int ldlq_ct_m359(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_241(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_462(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_146(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_58_299(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_211_397(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_ct_m359_40_475(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);
int ldlq_rt(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st);

}  // namespace ltqb
