// Traceback / reconstruction kernel instantiations (one per parity mode; label masks are run-time values here).
#include "vit_launch.cuh"
namespace ltqb {

template <int MD>
static int launch_tb_md(const VitParams& p, cudaStream_t st)
{
    const int smem = tb_smem(p.T, p.sub, p.nl, p.U, p.U_hi, p.W4, p.NB, TB_WARPS).total;
    auto k = vit_tb_kernel<MD>;
    static std::atomic<int> done[64];
    if (ensure_smem(k, smem, done) != 0) return -1;
    k<<<(p.N + TB_WARPS - 1) / TB_WARPS, 32 * TB_WARPS, smem, st>>>(p);
    return 0;
}

int launch_tb(const VitParams& p, int md, cudaStream_t st)
{
    switch (md) {
        case 0: return launch_tb_md<0>(p, st);
        case 1: return launch_tb_md<1>(p, st);
        case 2: return launch_tb_md<2>(p, st);
        case 3: return launch_tb_md<3>(p, st);
        default: return -1;
    }
}

}  // namespace ltqb
