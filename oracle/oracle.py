"""TEST INFRASTRUCTURE ONLY — the CPU oracle for the LTQ TCQ quantizer path; never part of the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import this module, and only as
the checker (or the timed CPU baseline).  The product path (``ltq_research_b200``) never imports it.

Contents, each restated from the reference (lumen-inference/ltq-research; paths relative to its root):

* ``viterbi``            — ``viterbi_ub_cuda`` (src/tcq_proto.py:567-657): the tail-biting schedule (:584-609) and the
                           return conventions (:653-657) over the C restatement of the kernel (oracle/tcq_oracle.c).
* ``LtqFormat`` …        — the format reference src/ltq_format.py:21-147 (labels, tile packing and decoding).
* ``pack_slice_regions`` / ``decode_slice_regions`` — src/ltq_file.py:54-148 (SoA regions on 64-byte boundaries).
* ``fwht``               — src/iqk_format.py:153-170 (normalized block FWHT, same butterfly order, fp32).
* ``lut_subs``           — src/cuda/tcq_viterbi.cu:768-804 (DP-profile sub-block quantization through the 1-D table).

Parity pins live in tests/test_oracle_golden.py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libtcq_oracle.so"
NU = 10
TILE = 256
MASK_M = 359

ROUND_FUSED = 7   # the reference CUDA kernel: x - g*tab and the candidate sum contracted into FMAs
ROUND_TORCH = 0   # the reference torch Viterbi on CPU: products rounded before the subtraction

_LIB = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.ora_tcq_viterbi.restype = ctypes.c_int
        L.ora_tcq_viterbi.argtypes = ([ctypes.c_void_p] * 15 + [ctypes.c_int] * 18 +
                                      [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int])
        L.ora_max_threads.restype = ctypes.c_int
        L.ora_lut_subs.restype = None
        L.ora_lut_subs.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int]
        _LIB = L
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def viterbi(x, small, K: int, nu: int, m: int, gains=None, sub: int = 16, wts=None, init_state=None,
            return_end_state: bool = False, small_hi=None, gains_hi=None, mix: int = 0, n_cand: int = 0,
            return_code: bool = False, tail_biting: bool = False, tb_passes: int = 2, tb_cand1: int = 0,
            tb_window: int = 0, m_extra: tuple = (), pair_parity=False, _mid: int = 0, _tail: bool = False,
            _steps: int = 0, _rot: int = 0, round_mode: int = ROUND_FUSED, n_threads: int = 0):
    """Oracle for ``viterbi_ub_cuda`` (src/tcq_proto.py:567-657) on numpy arrays; same arguments and return values."""
    x = _f32(x)
    if tail_biting:   # src/tcq_proto.py:584-609
        N, T = x.shape
        h = T // 2
        kw = dict(sub=sub, small_hi=small_hi, gains_hi=gains_hi, mix=mix, n_cand=n_cand, m_extra=m_extra,
                  pair_parity=pair_parity, round_mode=round_mode, n_threads=n_threads)
        w_full = None if wts is None else _f32(np.broadcast_to(np.asarray(wts, np.float32).reshape(-1, T), (N, T)))
        kw1 = dict(kw, n_cand=tb_cand1) if tb_cand1 else kw
        if tb_window:
            _, mid = viterbi(x, small, K, nu, m, gains, wts=w_full, _mid=tb_window, _steps=2 * tb_window,
                             _rot=h - tb_window, **kw1)
        else:
            _, mid = viterbi(x, small, K, nu, m, gains, wts=w_full, _mid=h, **kw1)
        shift = 0
        out = None
        for p in range(1, tb_passes):
            shift = (shift + h) % T
            if p + 1 < tb_passes:
                _, mid = viterbi(x, small, K, nu, m, gains, wts=w_full, init_state=mid, _tail=True, _mid=h,
                                 _rot=shift, **kw)
            else:
                out = viterbi(x, small, K, nu, m, gains, wts=w_full, init_state=mid, return_code=return_code,
                              _tail=True, _rot=shift, **kw)
        return out
    N, ld = x.shape
    T = _steps or ld
    S, U = 1 << nu, 1 << (K - 1)
    if wts is None:
        w = np.ones_like(x)
    else:
        w = _f32(np.broadcast_to(np.asarray(wts, np.float32).reshape(-1, ld), (N, ld)))
    g = _f32(gains if gains is not None else np.ones(1, np.float32))
    tab = _f32(small)
    rec = np.zeros_like(x)
    tab_hi = _f32(small_hi) if small_hi is not None else tab
    g_hi = _f32(gains_hi) if gains_hi is not None else g
    init = np.ascontiguousarray(np.asarray(init_state, dtype=np.int32)) if init_state is not None else None
    end = np.zeros(N, np.int32) if return_end_state else None
    Gfull = g.size
    best = np.zeros(N, np.int32)
    code = np.zeros((N, ld), np.int32) if return_code else None
    mid = np.zeros(N, np.int32) if _mid else None
    nl = 4 << len(m_extra)
    cand = np.zeros((N, T // sub, n_cand), np.uint8) if 0 < n_cand < Gfull else None
    me = (list(m_extra) + [0, 0, 0])[:3]
    rc = lib().ora_tcq_viterbi(_ptr(x), _ptr(w), _ptr(tab), _ptr(g), _ptr(rec), None, None, _ptr(init), _ptr(end),
                               _ptr(tab_hi), _ptr(g_hi), _ptr(cand), _ptr(best), _ptr(code), _ptr(mid), _mid,
                               int(_tail), N, T, S, U, n_cand if cand is not None else Gfull, Gfull, m, sub,
                               tab_hi.size // nl, mix if small_hi is not None else 0, me[0], me[1], me[2], nl, ld,
                               _rot, None, int(pair_parity), None, int(round_mode), int(n_threads))
    if rc != 0:
        raise RuntimeError(f"tcq_viterbi: CUDA error code {rc}")
    if _mid:
        return rec, mid
    if return_code:
        return rec, code >> 16, code & 0xFFFF
    return (rec, end) if return_end_state else rec


def make_gains(h: int, step: float) -> np.ndarray:
    """float64 evaluation of 2^((g - (G-1)/2) * step) rounded to fp32 (src/tcq_proto.py:247-249).  The format stores
    the exact fp32 values it was quantized with (src/ltq_format.py:31-32); tests take gains from their fixture."""
    G = 1 << h
    return (2.0 ** ((np.arange(G, dtype=np.float64) - (G - 1) / 2) * step)).astype(np.float32)


# ---------------------------------------------------------------------------------------------------------------
# Format reference restated: src/ltq_format.py
# ---------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class LtqFormat:
    """src/ltq_format.py:21-54."""
    name: str
    K: int
    frac: int
    masks: tuple
    h: int
    step: float
    sub: int
    lut: np.ndarray
    gain_tab: np.ndarray

    @property
    def n_labels(self) -> int:
        return 2 ** len(self.masks) * 2

    @property
    def U(self) -> int:
        return 1 << (self.K - 1)

    def lsb_words(self, L: int = TILE) -> int:
        return ({0: L, 1: L // 2, 2: 3 * L // 4}[self.frac] + 15) // 16

    def gain_words(self, L: int = TILE) -> int:
        return (L // self.sub * self.h + 15) // 16

    def tile_bytes(self, L: int = TILE) -> int:
        return 2 * (L // 16 + L // 16 * (self.K - 2) + (self.lsb_words(L) if self.K > 1 else 0) + self.gain_words(L))

    def bpw(self, k_in: int) -> float:
        return self.tile_bytes() * 8 / TILE + 8 / 256 + 16 / k_in


def parity(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x).astype(np.uint32)
    for s in (16, 8, 4, 2, 1):
        x = x ^ (x >> s)
    return x & 1


def states_from_codes(c: np.ndarray) -> np.ndarray:
    """src/ltq_format.py:76-84: s_t = sum_j c[(t - j) mod L] << j, j < 10."""
    L = len(c)
    t = np.arange(L)
    s = np.zeros(L, dtype=np.uint32)
    for j in range(NU):
        s |= np.asarray(c)[(t - j) % L].astype(np.uint32) << j
    return s


def labels_from_states(s: np.ndarray, fmt: LtqFormat) -> np.ndarray:
    """src/ltq_format.py:87-91."""
    lb = (s & 1) | (parity((s >> 1) & fmt.masks[0]) << 1)
    for i, m in enumerate(fmt.masks[1:]):
        lb |= parity((s >> 1) & m) << (2 + i)
    return lb


def _bits_to_words(bits: np.ndarray, n_words: int) -> np.ndarray:
    out = np.zeros(n_words * 16, dtype=np.uint32)
    out[: len(bits)] = bits
    return (out.reshape(n_words, 16) << np.arange(16, dtype=np.uint32)).sum(axis=1).astype(np.uint16)


def _words_to_bits(words: np.ndarray, n_bits: int) -> np.ndarray:
    return ((np.asarray(words).astype(np.uint32)[:, None] >> np.arange(16, dtype=np.uint32)) & 1).reshape(-1)[:n_bits]


def pack_tile(labels: np.ndarray, u: np.ndarray, gidx: np.ndarray, fmt: LtqFormat) -> dict:
    """src/ltq_format.py:104-123."""
    labels = np.asarray(labels).astype(np.uint32)
    u = np.asarray(u).astype(np.uint32)
    L = len(labels)
    W = L // 16
    codes = _bits_to_words(labels & 1, W)
    planes = (np.stack([_bits_to_words((u >> p) & 1, W) for p in range(1, fmt.K - 1)]) if fmt.K > 2
              else np.zeros((0, W), np.uint16))
    lsb_all = u & 1
    if fmt.frac == 0:
        lsb = _bits_to_words(lsb_all, fmt.lsb_words(L))
    elif fmt.frac == 1:
        lsb = _bits_to_words(lsb_all[0::2], fmt.lsb_words(L))
    else:
        lsb = _bits_to_words(lsb_all.reshape(-1, 4)[:, :3].reshape(-1), fmt.lsb_words(L))
    g = np.asarray(gidx)[:: fmt.sub].astype(np.uint32)
    gbits = ((g[:, None] >> np.arange(fmt.h, dtype=np.uint32)) & 1).reshape(-1) if fmt.h else np.zeros(0, np.uint32)
    return {"L": L, "codes": codes, "planes": planes, "lsb": lsb,
            "gains": _bits_to_words(gbits, fmt.gain_words(L)) if fmt.h else np.zeros(0, np.uint16)}


def decode_tile(f: dict, fmt: LtqFormat) -> np.ndarray:
    """src/ltq_format.py:126-147."""
    L = f.get("L", TILE)
    c = _words_to_bits(f["codes"], L)
    lb = labels_from_states(states_from_codes(c), fmt)
    if fmt.frac == 0:
        lsb = _words_to_bits(f["lsb"], L)
    elif fmt.frac == 1:
        lsb = np.repeat(_words_to_bits(f["lsb"], L // 2), 2)
    else:
        b3 = _words_to_bits(f["lsb"], 3 * L // 4).reshape(-1, 3)
        lsb = np.concatenate([b3, (b3.sum(axis=1, keepdims=True) & 1)], axis=1).reshape(-1)
    u = lsb.copy()
    for p in range(1, fmt.K - 1):
        u |= _words_to_bits(f["planes"][p - 1], L) << p
    if fmt.h:
        gb = _words_to_bits(f["gains"], L // fmt.sub * fmt.h).reshape(-1, fmt.h)
        g = (gb << np.arange(fmt.h, dtype=np.uint32)).sum(axis=1)
        gain = fmt.gain_tab[np.repeat(g, fmt.sub)]
    else:
        gain = np.ones(L, dtype=np.float32)
    return (gain * fmt.lut[lb * fmt.U + u]).astype(np.float32)


def tile_words(f: dict) -> np.ndarray:
    """Concatenated u16 fields of one packed tile in spec order (codes, planes, lsb, gains)."""
    return np.concatenate([f["codes"], np.asarray(f["planes"]).reshape(-1), f["lsb"], f["gains"]]).astype(np.uint16)


# ---------------------------------------------------------------------------------------------------------------
# .ltq slice regions restated: src/ltq_file.py:54-148
# ---------------------------------------------------------------------------------------------------------------

def _align(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def tiles(x: np.ndarray) -> np.ndarray:
    """src/ltq_file.py:69-72: [R, K] -> [T, 256], tiles by row group then by 16-column block; t = 16 r + c."""
    R, K = x.shape
    return x.reshape(R // 16, 16, K // 16, 16).transpose(0, 2, 1, 3).reshape(-1, TILE)


def untiles(t: np.ndarray, R: int, K: int) -> np.ndarray:
    return t.reshape(R // 16, K // 16, 16, 16).transpose(0, 2, 1, 3).reshape(R, K)


def pack_slice(idx: np.ndarray, gi: np.ndarray, f: LtqFormat) -> bytes:
    """src/ltq_file.py:79-102: four SoA regions (codes, planes, lsb, gains), each starting on a 64-byte boundary."""
    ix, g = tiles(np.asarray(idx).astype(np.int64)), tiles(np.asarray(gi).astype(np.int64))
    T = ix.shape[0]
    lab, u = ix // f.U, ix % f.U

    def words(bits):
        n = bits.shape[1]
        n16 = _align(n, 16)
        if n16 != n:
            bits = np.concatenate([bits, np.zeros((T, n16 - n), bits.dtype)], axis=1)
        return (bits.reshape(T, -1, 16).astype(np.int64) << np.arange(16)).sum(axis=2)

    regions = [words(lab & 1)]
    regions.append(np.stack([words((u >> p) & 1) for p in range(1, f.K - 1)], axis=1).reshape(T, -1) if f.K > 2
                   else np.zeros((T, 0), np.int64))
    lsb = u & 1
    if f.frac == 1:
        lsb = lsb[:, 0::2]
    elif f.frac == 2:
        lsb = lsb.reshape(T, -1, 4)[:, :, :3].reshape(T, -1)
    regions.append(words(lsb))
    if f.h:
        gs = g[:, :: f.sub]
        regions.append(words(((gs[:, :, None] >> np.arange(f.h)) & 1).reshape(T, -1)))
    else:
        regions.append(np.zeros((T, 0), np.int64))
    out = bytearray()
    for r in regions:
        out += bytes(_align(len(out), 64) - len(out))
        out += r.astype(np.uint16).tobytes()
    return bytes(out)


def decode_slice(data: bytes, R: int, K: int, f: LtqFormat) -> np.ndarray:
    """src/ltq_file.py:119-148: unscaled slice values [R, K] from the SoA bytes, by the spec."""
    T = (R // 16) * (K // 16)
    sizes = [16, 16 * (f.K - 2), f.lsb_words(), f.gain_words()]
    regions, off = [], 0
    for n in sizes:
        off = _align(off, 64)
        regions.append(np.frombuffer(data[off: off + 2 * T * n], dtype=np.uint16).reshape(T, n) if n else None)
        off += 2 * T * n

    def bits(words, n):
        return ((words.astype(np.int64)[:, :, None] >> np.arange(16)) & 1).reshape(words.shape[0], -1)[:, :n]

    c = bits(regions[0], TILE)
    s = sum(np.roll(c, j, axis=1) << j for j in range(NU))
    lab = labels_from_states(s.astype(np.uint32), f).astype(np.int64)
    lb = bits(regions[2], {0: TILE, 1: TILE // 2, 2: 3 * TILE // 4}[f.frac])
    if f.frac == 1:
        lb = np.repeat(lb, 2, axis=1)
    elif f.frac == 2:
        b3 = lb.reshape(T, -1, 3)
        lb = np.concatenate([b3, b3.sum(axis=2, keepdims=True) & 1], axis=2).reshape(T, TILE)
    u = lb
    for p in range(1, f.K - 1):
        u = u | (bits(regions[1][:, 16 * (p - 1): 16 * p], TILE) << p)
    if f.h:
        gb = bits(regions[3], TILE // f.sub * f.h).reshape(T, -1, f.h)
        g = np.repeat((gb << np.arange(f.h)).sum(axis=2), f.sub, axis=1)
        gain = f.gain_tab[g]
    else:
        gain = np.ones((T, TILE), np.float32)
    vals = (gain * f.lut[lab * f.U + u]).astype(np.float32)
    return untiles(vals, R, K)


# ---------------------------------------------------------------------------------------------------------------
# FWHT restated: src/iqk_format.py:153-170
# ---------------------------------------------------------------------------------------------------------------

def fwht(x: np.ndarray, block_size: int = 256) -> np.ndarray:
    """Normalized block FWHT over the last dim, fp32: stages h = 1, 2, ..., block/2 of (a + b, a - b) on pairs
    (i, i + h) within each 2h-group, then one multiply by block^-0.5."""
    x = np.asarray(x, dtype=np.float32)
    shp = x.shape
    y = x.reshape(-1, block_size).copy()
    h = 1
    while h < block_size:
        v = y.reshape(-1, block_size // (2 * h), 2, h)
        a = v[:, :, 0, :].copy()
        b = v[:, :, 1, :].copy()
        v[:, :, 0, :] = a + b
        v[:, :, 1, :] = a - b
        y = v.reshape(-1, block_size)
        h *= 2
    return (y.reshape(shp) * np.float32(block_size ** -0.5)).astype(np.float32)


def max_threads() -> int:
    return int(lib().ora_max_threads())


if __name__ == "__main__":
    build()
    print(LIB_PATH, os.path.getsize(LIB_PATH), "bytes,", max_threads(), "threads")


def lut_subs(xs, dh, lut, inv_step: float, half_b: float) -> np.ndarray:
    """lut_subs_quant (src/cuda/tcq_viterbi.cu:768-811) on CPU: xs, dh [S, 16], lut [nb, 64] -> [S, 16]."""
    x = _f32(xs).reshape(-1, 16)
    d = _f32(dh).reshape(x.shape)
    t = _f32(lut)
    assert t.ndim == 2 and t.shape[1] == 64
    out = np.empty_like(x)
    lib().ora_lut_subs(_ptr(x), _ptr(d), _ptr(t), _ptr(out), x.shape[0], float(inv_step), float(half_b), t.shape[0])
    return out
