// Viterbi kernel instantiation: label masks (359, 0, 0, 0), 4 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int launch_ct_m359(const VitParams& p, int md, int smem, cudaStream_t st)
{
    return launch_md<MaskCT<359, 0, 0, 0, 4>>(p, md, smem, st);
}
}  // namespace ltqb
