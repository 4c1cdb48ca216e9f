"""Golden outputs of the reference's own DP-profile kernel (lut_subs_quant, src/cuda/tcq_viterbi.cu:768-811), compiled
from the reference source for sm_100a (oracle/_ref, `make -C oracle ref`) and run on a B200 on the seeded inputs of
tests/golden/lut_inputs.py.  Run on a GPU box:  python tests/golden/make_golden_lut.py [OUT]
(default OUT: tests/golden/lut_subs.npz)."""
import ctypes
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from tests.golden.lut_inputs import case  # noqa: E402


def main():
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libtcq_viterbi_ref.so"))
    lib.lut_subs_quant.restype = ctypes.c_int
    lib.lut_subs_quant.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                           ctypes.c_void_p]
    xs, dh, lut, inv_step, half_b = case()
    dev = torch.device("cuda", 0)
    x, d, t = (torch.from_numpy(a).to(dev).contiguous() for a in (xs, dh, lut))
    out = torch.empty_like(x)
    rc = lib.lut_subs_quant(x.data_ptr(), d.data_ptr(), t.data_ptr(), out.data_ptr(), x.shape[0], inv_step, half_b,
                            t.shape[0], torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, rc
    dst = Path(sys.argv[1]) if len(sys.argv) > 1 else ROOT / "tests" / "golden" / "lut_subs.npz"
    np.savez_compressed(dst, out=out.cpu().numpy())
    print(dst, out.shape)


if __name__ == "__main__":
    main()
