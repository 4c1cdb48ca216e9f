// Fused LDLQ block instantiation: label masks (359, 241, 0, 0), 8 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int ldlq_ct_m359_241(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st)
{
    return launch_ldlq_md<MaskCT<359, 241, 0, 0, 8>>(q, md, smem, grid, st);
}
}  // namespace ltqb
