"""ltq_research_b200 — the LTQ TCQ quantizer hot path on NVIDIA B200 (sm_100a).

Public API (mirrors lumen-inference/ltq-research):
  * ``tcq_proto.viterbi_ub_cuda`` / ``viterbi_ub`` / ``make_gains`` — src/tcq_proto.py
  * ``formats.TCQ_CONFIG`` / ``LIQK_V2_SPECS`` / ``SETS`` / ``LtqFormat`` / ``load_formats`` — src/liqk_v2.py,
    src/equal_bpw.py, src/ltq_format.py
The CUDA kernels live in ``libltq_b200.so`` (C ABI: include/ltq_b200.h), built by ``python -m ltq_research_b200.build``.
"""
from .tcq_proto import make_gains, viterbi_ub, viterbi_ub_cuda  # noqa: F401

__version__ = "0.1.0"
