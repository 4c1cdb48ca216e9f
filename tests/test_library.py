"""The C-ABI library loads, exports every entry point include/*.h declares, and validates arguments exactly as the
reference does (returns -1 before touching a GPU).  No GPU needed."""
import re
from pathlib import Path

import pytest

from ltq_research_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_header_symbols():
    L = _lib.lib()
    declared = _declared()
    assert "tcq_viterbi" in declared and "ltq_viterbi_tb" in declared
    for name in declared:
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.SIGNATURES"
    assert L.ltq_b200_version().decode().startswith("ltq_b200")


def _call(**over):
    # a valid config-1 call (K = 2, 4 subsets, 4 gains, sub = 16, T = 256); pointers are never touched on -1
    a = dict(x=None, w=None, tab=None, gains=None, rec=None, bp=None, gsel=None, init_st=None, end_st=None, tab_hi=None,
             gains_hi=None, gcand=None, best=None, code=None, mid_st=None, mid_t=0, tail=0, N=4, T=256, S=1024, U=2, G=4,
             Gfull=4, m=359, sub=16, U_hi=2, mix=0, m2=0, m3=0, m4=0, nl=4, ld=256, rot=0, pbits=None, pp=0,
             stream=None)
    a.update(over)
    return _lib.lib().tcq_viterbi(*a.values())


@pytest.mark.parametrize("over", [
    dict(G=5, Gfull=5), dict(G=17, Gfull=17), dict(Gfull=8),           # G set, candidates need gcand
    dict(U=129), dict(U_hi=129), dict(sub=15), dict(sub=6),             # U, odd sub, T % sub
    dict(T=1024, ld=1024), dict(sub=64, T=256), dict(T=512, ld=512, sub=8),  # T > 512, sub > 32, T / sub > 32
    dict(pp=1, mix=16), dict(pp=2, sub=18, T=252, ld=252), dict(pp=4),   # parity-mode limits
    dict(nl=12), dict(ld=128), dict(S=256, nl=8), dict(nl=32, U=32),    # labels, row stride, table size
    dict(G=8, Gfull=8, nl=16, sub=32, pp=1),                             # sub * G * nl * NP > 4096
])
def test_validation_matches_reference(over):
    assert _call(**over) == -1


def test_state_and_subset_limits():
    """The 256-state trellis and 32 label subsets are accepted (GPU tests check them); what the reference's table
    rejects around them is rejected before any launch: 256 states with a parity mode or extra subsets, other state
    counts, 32 subsets with too wide a table or too many slot x step x label errors."""
    assert _call(S=256, pp=1) == -1
    assert _call(S=256, nl=16, m2=5, m3=9) == -1
    assert _call(S=512) == -1 and _call(S=2048) == -1
    assert _call(nl=32, U=32) == -1
    assert _call(nl=32, U=2, G=8, Gfull=8, sub=32) == -1


def test_workspace_size():
    L = _lib.lib()
    b = L.ltq_viterbi_tb_workspace_bytes(65536, 256, 4, 0, 16, 0, 0, 0)
    # survivors: 64 groups x 2 words x 32 lanes x 4 B per slot -> 16 KiB per slot, 4 slots
    assert b >= 65536 * 4 * 16384
    assert b < 65536 * 4 * 16384 * 1.15  # + gain-merge winners: 16 boundaries x 512 B per tile
    assert L.ltq_viterbi_tb_workspace_bytes(0, 256, 4, 0, 16, 0, 0, 0) == 0


def test_no_cpu_fallback():
    import torch
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    x = torch.zeros(2, 256)
    with pytest.raises(RuntimeError, match="CUDA"):
        viterbi_ub_cuda(x, torch.zeros(8), 2, 10, 359)


def test_matrix_entries_reject_bad_arguments():
    """The Hessian and LDLQ helper entry points return -1 on invalid sizes, strides and alignments before any CUDA
    call (fake, never-dereferenced addresses)."""
    L = _lib.lib()
    a, b = 1 << 20, 1 << 21  # 16-byte aligned stand-ins
    # blocked-Cholesky diagonal step: null pointers, c0 or ld not a multiple of 4, ld too small, misaligned pointers
    assert L.ltq_chol256_diag(None, 256, 0, b, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 256, 0, None, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 256, 0, b, None, 0, None, None) == -1
    assert L.ltq_chol256_diag(a, 512, 2, b, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 254, 0, b, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 510, 256, b, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a + 4, 256, 0, b, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 256, 0, b + 2, None, 0, a, None) == -1
    assert L.ltq_chol256_diag(a, 256, 0, b, a, 255, a, None) == -1
    # six-slot operand split: bad order / side, unaligned input, output row stride too small
    assert L.ltq_bf16x6_split(a, 256, 4, 256, 2, 0, b, 1536, None) == -1
    assert L.ltq_bf16x6_split(a, 256, 4, 256, 0, 2, b, 1536, None) == -1
    assert L.ltq_bf16x6_split(a + 4, 256, 4, 256, 0, 0, b, 1536, None) == -1
    assert L.ltq_bf16x6_split(a, 256, 4, 256, 0, 0, b, 1532, None) == -1
