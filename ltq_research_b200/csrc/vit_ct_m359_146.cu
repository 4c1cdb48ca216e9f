// Viterbi kernel instantiation: label masks (359, 146, 0, 0), 8 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int launch_ct_m359_146(const VitParams& p, int md, int smem, cudaStream_t st)
{
    return launch_md<MaskCT<359, 146, 0, 0, 8>>(p, md, smem, st);
}
}  // namespace ltqb
