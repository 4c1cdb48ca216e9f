// Viterbi kernel instantiation for label masks given at run time (4, 8, 16 or 32 subsets).
#include "vit_launch.cuh"
namespace ltqb {
int launch_rt(const VitParams& p, int md, int smem, cudaStream_t st)
{
    switch (p.nl) {
        case 4: return launch_md<MaskRT<4>>(p, md, smem, st);
        case 8: return launch_md<MaskRT<8>>(p, md, smem, st);
        case 16: return launch_md<MaskRT<16>>(p, md, smem, st);
        case 32: return launch_md<MaskRT<32>>(p, md, smem, st);
        default: return -1;
    }
}
int launch_rt_sub2(const VitParams& p, int md, int smem, cudaStream_t st)
{
    switch (p.nl) {
        case 4: return launch_md_sub2<MaskRT<4>>(p, md, smem, st);
        case 8: return launch_md_sub2<MaskRT<8>>(p, md, smem, st);
        case 16: return launch_md_sub2<MaskRT<16>>(p, md, smem, st);
        case 32: return launch_md_sub2<MaskRT<32>>(p, md, smem, st);
        default: return -1;
    }
}
}  // namespace ltqb
