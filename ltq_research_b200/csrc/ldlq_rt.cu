// Fused LDLQ block instantiation for label masks given at run time (4, 8 or 16 subsets).
#include "vit_launch.cuh"
namespace ltqb {
int ldlq_rt(const LdlqParams& q, int md, int smem, int grid, cudaStream_t st)
{
    switch (q.p2.nl) {
        case 4: return launch_ldlq_md<MaskRT<4>>(q, md, smem, grid, st);
        case 8: return launch_ldlq_md<MaskRT<8>>(q, md, smem, grid, st);
        case 16: return launch_ldlq_md<MaskRT<16>>(q, md, smem, grid, st);
        default: return -1;
    }
}
}  // namespace ltqb
