// Viterbi kernel instantiation: label masks (359, 462, 0, 0), 8 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int launch_ct_m359_462(const VitParams& p, int md, int smem, cudaStream_t st)
{
    return launch_md<MaskCT<359, 462, 0, 0, 8>>(p, md, smem, st);
}
}  // namespace ltqb
