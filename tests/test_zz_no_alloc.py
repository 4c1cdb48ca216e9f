"""The allocation-free tail-biting Viterbi (ltq_viterbi_tb_noalloc) against the workspace entry point (ltq_viterbi_tb).

Some callers cannot allocate device memory while they quantize (an engine that plans its device memory at start-up,
or a binding that only holds device pointers to its inputs and outputs); for them the library keeps the scratch in a
fixed 64 MiB array of its own.  This test calls both entry points through the C ABI on the same inputs, two calls in a
row with different formats and inputs (the second call finds the first call's leftovers in the shared array), and
requires identical results.  It sits in its own file so that it runs last.
"""
import ctypes

import numpy as np
import pytest
import torch

from ltq_research_b200 import _lib
from tests import vit_cases as VC

pytestmark = pytest.mark.gpu


def _args(name, N, seed, dev):
    c = VC.F[name]
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(N, 256, generator=g).to(dev)
    w = (torch.rand(256, generator=g) * 2 + 0.1).to(dev)
    lut = torch.tensor(c["lut"], dtype=torch.float32, device=dev)
    gains = torch.tensor(c["gains_cpu"], dtype=torch.float32, device=dev)
    me = np.asarray(list(c["m_extra"]) + [0], dtype=np.int32)
    return c, x, w, lut, gains, me


def _run(entry, name, N, seed, dev, window=32):
    L = _lib.lib()
    c, x, w, lut, gains, me = _args(name, N, seed, dev)
    rec = torch.empty_like(x)
    code = torch.empty(x.shape, dtype=torch.int32, device=dev)
    common = [x.data_ptr(), w.data_ptr(), 0, lut.data_ptr(), gains.data_ptr(), None, None, rec.data_ptr(),
              code.data_ptr(), N, 256, 10, c["K"], c["m"], me.ctypes.data_as(ctypes.c_void_p), len(c["m_extra"]),
              gains.numel(), c["n_cand"], c["sub"], 1 << (c["K"] - 1), 0, c["pp"], 2, 0, window]
    stream = torch.cuda.current_stream(dev).cuda_stream
    if entry == "workspace":
        wsb = L.ltq_viterbi_tb_workspace_bytes(N, 256, gains.numel(), c["n_cand"], c["sub"], c["pp"], window, 0)
        ws = torch.empty(int(wsb), dtype=torch.uint8, device=dev)
        rc = L.ltq_viterbi_tb(*common, ws.data_ptr(), ws.numel(), stream)
    else:
        rc = L.ltq_viterbi_tb_noalloc(*common, stream)
    torch.cuda.synchronize()
    assert rc == 0, rc
    return rec.cpu().numpy(), code.cpu().numpy()


def test_noalloc_matches_workspace_entry_two_calls(cuda_dev):
    # two calls in a row: a D2 format, then a plain one with different tiles; both must equal the workspace entry
    for name, N, seed in (("TCQ25X", 96, 1), ("TCQ3X", 160, 2)):
        want = _run("workspace", name, N, seed, cuda_dev)
        got = _run("noalloc", name, N, seed, cuda_dev)
        assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32)), name
        assert np.array_equal(got[1], want[1]), name


def test_noalloc_rejects_requests_beyond_capacity(cuda_dev):
    L = _lib.lib()
    cap = L.ltq_viterbi_tb_noalloc_capacity()
    assert cap == 64 << 20
    N = 4096  # 4096 tiles x 4 slots x 16 KiB of survivor words > 64 MiB
    assert L.ltq_viterbi_tb_workspace_bytes(N, 256, 4, 0, 16, 0, 0, 0) > cap
    rc = L.ltq_viterbi_tb_noalloc(None, None, 0, None, None, None, None, None, None, N, 256, 10, 2, 359, None, 0, 4, 0,
                                  16, 2, 0, 0, 2, 0, 0, None)
    assert rc == -2
