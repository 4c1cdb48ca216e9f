// Fused LDLQ block instantiation: label masks (359, 58, 299, 0), 16 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int ldlq_ct_m359_58_299(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st)
{
    return launch_ldlq_md<MaskCT<359, 58, 299, 0, 16>>(q, md, smem, grid, st);
}
}  // namespace ltqb
