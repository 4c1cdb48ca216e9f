// Fused LDLQ block instantiation: label masks (359, 40, 475, 0), 16 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int ldlq_ct_m359_40_475(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st)
{
    return launch_ldlq_md<MaskCT<359, 40, 475, 0, 16>>(q, md, smem, grid, st);
}
}  // namespace ltqb
