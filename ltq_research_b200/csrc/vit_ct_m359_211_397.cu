// Viterbi kernel instantiation: label masks (359, 211, 397, 0), 16 subsets.
#include "vit_launch.cuh"
namespace ltqb {
int launch_ct_m359_211_397(const VitParams& p, int md, int smem, cudaStream_t st)
{
    return launch_md<MaskCT<359, 211, 397, 0, 16>>(p, md, smem, st);
}
}  // namespace ltqb
