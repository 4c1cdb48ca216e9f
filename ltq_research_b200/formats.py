"""LTQ tile formats: the reference's format menu and format description.

Mirrors lumen-inference/ltq-research:
  * ``TCQ_CONFIG`` / ``TCQ_X_SCALE`` for the tail-biting (.ltq) formats — src/liqk_v2.py:818-840 (tables from
    results/tcq_x_tables.json, n_cand = 4 when h > 2) — and the earlier formats of src/liqk_v2.py:786-821;
  * ``LIQK_V2_SPECS`` bit accounting of those formats — src/liqk_v2.py:862-869;
  * ``SETS`` format menus (``TCQPQ`` = the 19-format menu) — src/equal_bpw.py:58-75;
  * ``LtqFormat`` / ``load_formats`` — src/ltq_format.py:21-66.
The format constants (LUTs, masks, gain steps, scales) live in data/tcq_formats.json; they define the format and are
identical to the reference's, or files would not be compatible.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Optional

import numpy as np
import torch

from .tcq_proto import make_gains

NU = 10          # trellis memory: state = last 10 code bits
TILE = 256       # weights per tile (16 x 16)
MASK_M = 359     # primary Ungerboeck label mask
QK_K = 256       # block of the scale exponent and of the FWHT rotation
SUBBLOCK_SIZE = 16

_DATA = json.loads((Path(__file__).resolve().parent / "data" / "tcq_formats.json").read_text())
SETS: Dict[str, list] = {k: list(v) for k, v in _DATA["sets"].items()}
MENU_TCQPQ: list = list(_DATA["menu_TCQPQ"])

TCQ_CONFIG: Dict[str, dict] = {}
TCQ_X_SCALE: Dict[str, float] = {}
for _name, _t in _DATA["formats"].items():
    if _name.startswith("_"):
        continue
    TCQ_CONFIG[_name] = {"K": _t["K"], "nu": _t["nu"], "m": _t["m"], "h": _t["h"], "step": _t["step"],
                         "lut": list(_t["lut"]), "sub": _t["sub"], "pp": _t["pp"], "scale": _t["scale"],
                         "m_extra": tuple(_t["m_extra"]), "row_scale": True, "tb": True,
                         **({"n_cand": 4} if _t["h"] > 2 else {})}
    TCQ_X_SCALE[_name] = _t["scale"]
# The earlier formats (src/liqk_v2.py:786-821), not tail-biting and not written to .ltq files: TCQ2 / TCQ3 / TCQ4 take a
# scale per (row, 256-block) refitted over two passes; the R formats one scale per row with 5-bit block exponents and the
# trellis state carried from each tile to the next tile of the same rows (one pass); TCQ25R / TCQ35R alternate tile rows
# between the tables of their "lo" and "hi" formats (each premultiplied by its own scale).
LEGACY_FORMATS: list = list(_DATA["legacy"])
for _name, _t in _DATA["legacy"].items():
    _c = {k: _t[k] for k in ("K", "nu", "m", "h", "scale")}
    if _t["row_scale"]:
        _c["row_scale"] = True
    if _t["carry"]:
        _c["carry"] = True
    if _t["n_cand"]:
        _c["n_cand"] = _t["n_cand"]
    if "K_hi" in _t:
        _c.update({"K_hi": _t["K_hi"], "lo": _t["lo"], "hi": _t["hi"]})
    else:
        _c.update({"step": _t["step"], "lut": list(_t["lut"])})
    TCQ_CONFIG[_name] = _c
# the tail-biting (.ltq) formats
LTQ_FORMATS: list = [n for n, c in TCQ_CONFIG.items() if c.get("tb")]
# config-1 Gaussian rig format (results/universal_gaussian.json "tcq_K2_h2": K = 2, 4 subsets, h = 2)
GAUSSIAN_RIG_K2H2: dict = dict(_DATA["formats"]["_config1_tcq_K2_h2"])


@dataclass(frozen=True)
class LiqkV2Spec:
    """src/liqk_v2.py:77-93 (only the fields the TCQ path uses)."""
    name: str
    bits: float
    n_levels: int
    n_pos_states: int
    block_bytes: float

    @property
    def bpw(self) -> float:
        return (self.block_bytes * 8.0) / QK_K


def _block_bits(c: dict) -> float:
    """Bits per 256 weights (src/liqk_v2.py:862-867): row-scale formats pay K (+ 1/2 for half-integer rows, minus the
    parity mode's saving) per weight, h per sub-block, 5 for the block exponent and 2 for the row scale's share; the
    block-scale formats pay the initial state (nu), a 16-bit scale and h per tile row."""
    if c.get("row_scale"):
        return (QK_K * (c["K"] + 0.5 * ("K_hi" in c) - {0: 0.0, 1: 0.5, 2: 0.25, 3: 0.75}[int(c.get("pp", 0))])
                + QK_K // c.get("sub", SUBBLOCK_SIZE) * c["h"] + 5 + 2)
    return QK_K * c["K"] + c["nu"] + 16 + 16 * c["h"]


LIQK_V2_SPECS: Dict[str, LiqkV2Spec] = {}
for _name, _cfg in TCQ_CONFIG.items():
    LIQK_V2_SPECS[_name] = LiqkV2Spec(_name, float(_cfg["K"]), 1 << (_cfg["K"] + 1), 1 << _cfg["h"],
                                      _block_bits(_cfg) / 8)


@dataclass(frozen=True)
class LtqFormat:
    """src/ltq_format.py:21-54: one tile format of the .ltq file."""
    name: str
    K: int
    frac: int           # 0 none, 1 D2 (K - 0.5), 2 D4 (K - 0.25), 3 EQ (K - 0.75)
    masks: tuple        # (m, *m_extra)
    h: int
    step: float
    sub: int
    lut: np.ndarray     # float32 [n_labels * 2^(K-1)], label-major
    gain_tab: np.ndarray  # float32 [2^h], stored explicitly in the file

    @property
    def n_labels(self) -> int:
        return 2 ** len(self.masks) * 2

    @property
    def U(self) -> int:
        return 1 << (self.K - 1)

    def lsb_words(self, L: int = TILE) -> int:
        return ({0: L, 1: L // 2, 2: 3 * L // 4, 3: L // 4}[self.frac] + 15) // 16

    def gain_words(self, L: int = TILE) -> int:
        return (L // self.sub * self.h + 15) // 16

    def tile_bytes(self, L: int = TILE) -> int:
        return 2 * (L // 16 + L // 16 * (self.K - 2) + (self.lsb_words(L) if self.K > 1 else 0) + self.gain_words(L))

    def bpw(self, k_in: int) -> float:
        return self.tile_bytes() * 8 / TILE + 8 / 256 + 16 / k_in


def load_formats(menu: list, device: Optional[torch.device | str] = None) -> Dict[str, LtqFormat]:
    """src/ltq_format.py:57-66.  Gains are evaluated by torch on ``device`` (default: the current CUDA device), as the
    reference does, because the rounding of 2^x differs between devices and the file stores the exact values."""
    dev = device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu")
    out = {}
    for name in menu:
        c = TCQ_CONFIG[name]
        out[name] = LtqFormat(name, c["K"], int(c.get("pp", 0)), (c["m"],) + tuple(c.get("m_extra", ())), c["h"],
                              float(c["step"]), c.get("sub", 16), np.asarray(c["lut"], dtype=np.float32),
                              make_gains(c["h"], c["step"], dev).cpu().numpy())
    return out
