"""The .ltq container on B200: packing, on-device verify, writing and reading (lumen-inference/ltq-research
src/ltq_file.py, same names, arguments and file layout).

Packing and the spec decode run as CUDA kernels (ltq_pack_slice / ltq_decode_slice of libltq_b200.so): the quantizer's
codes never leave the device until the packed bytes do, and LtqWriter.add_matrix verifies every slice on the device
(decode of the packed bytes against the quantizer's tile values, bit for bit) before writing it.

    python -m ltq_research_b200.ltq_file --check model.ltq
"""
from __future__ import annotations

import argparse
import ctypes
import json
import struct
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import ptr
from .formats import TILE, LtqFormat

MAGIC = b"LTQ\0"
VERSION = 1
DTYPES = {"f32": (np.float32, torch.float32), "f16": (np.float16, torch.float16), "bf16": (np.uint16, torch.bfloat16),
          "i32": (np.int32, torch.int32), "i8": (np.int8, torch.int8), "u8": (np.uint8, torch.uint8)}
TORCH_TO_LTQ = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16", torch.int32: "i32", torch.int8: "i8",
                torch.uint8: "u8"}
FRAC_NAMES = ["none", "d2", "d4"]


def _align(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def format_json(f: LtqFormat) -> dict:
    """Format description for the header (src/ltq_file.py:39-43): lut and gain as float32 values."""
    if f.frac >= len(FRAC_NAMES):
        raise ValueError(f"{f.name}: fractional mode {f.frac} has no .ltq encoding")
    return {"name": f.name, "K": f.K, "frac": FRAC_NAMES[f.frac], "masks": [int(m) for m in f.masks], "h": f.h,
            "sub": f.sub, "lut": [float(v) for v in np.asarray(f.lut, np.float32)],
            "gain": [float(v) for v in np.asarray(f.gain_tab, np.float32)]}


def format_from_json(d: dict) -> LtqFormat:
    return LtqFormat(d["name"], d["K"], FRAC_NAMES.index(d["frac"]), tuple(d["masks"]), d["h"], 0.0, d["sub"],
                     np.asarray(d["lut"], np.float32), np.asarray(d["gain"], np.float32))


def _check_fmt(f: LtqFormat):
    if f.frac >= len(FRAC_NAMES):
        raise ValueError(f"{f.name}: fractional mode {f.frac} has no .ltq encoding")


def slice_bytes(R: int, K: int, f: LtqFormat) -> int:
    """Bytes of a packed row slice [R, K] of format f."""
    _check_fmt(f)
    n = int(_lib.lib().ltq_slice_bytes(R, K, f.K, f.frac, f.h, f.sub))
    if n == 0 and R * K:
        raise ValueError(f"{f.name}: unsupported slice {R} x {K}")
    return n


def pack_slice_device(idx: torch.Tensor, gi: torch.Tensor, f: LtqFormat,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The packed bytes of a row slice as a uint8 CUDA tensor (src/ltq_file.py:79-102 computed on the device).
    idx (label * U + u) int16 and gi uint8 [R, K] CUDA tensors (a row range of the quantizer's PACK fields)."""
    dev = _lib.require_cuda(idx, gi)
    R, K = idx.shape
    if idx.dtype != torch.int16:
        idx = idx.to(torch.int16)
    if gi.dtype != torch.uint8:
        gi = gi.to(torch.uint8)
    if idx.stride(1) != 1 or gi.stride(1) != 1 or idx.stride(0) != gi.stride(0) or idx.stride(0) % 8:
        idx, gi = idx.contiguous(), gi.contiguous()
    n = slice_bytes(R, K, f)
    if out is None:
        out = torch.empty(_align(max(n, 1), 64), dtype=torch.uint8, device=dev)
    rc = _lib.lib().ltq_pack_slice(ptr(idx), ptr(gi), idx.stride(0), R, K, f.K, f.frac, f.h, f.sub, ptr(out),
                                   out.numel(), _lib.stream_ptr(dev))
    if rc != 0:
        raise RuntimeError(f"ltq_pack_slice: error code {rc}")
    return out[:n]


def pack_slice(idx: torch.Tensor, gi: torch.Tensor, f: LtqFormat) -> bytes:
    """src/ltq_file.py:79-102: four SoA regions (codes, planes, lsb, gains) on 64-byte boundaries, as bytes."""
    return bytes(pack_slice_device(idx, gi, f).cpu().numpy().tobytes())


_FMT_TABLES: Dict[tuple, tuple] = {}


def _tables(f: LtqFormat, device) -> tuple:
    """(lut, gain_tab) of a format as device tensors, cached per (format values, device)."""
    dev = torch.device(device)
    key = (f.name, str(dev), np.asarray(f.lut, np.float32).tobytes(), np.asarray(f.gain_tab, np.float32).tobytes())
    t = _FMT_TABLES.get(key)
    if t is None:
        t = (torch.as_tensor(np.asarray(f.lut, np.float32)).to(dev),
             torch.as_tensor(np.asarray(f.gain_tab, np.float32).reshape(-1)).to(dev))
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
        _FMT_TABLES[key] = t
    return t


def decode_slice_device(data: torch.Tensor, R: int, K: int, f: LtqFormat, out: Optional[torch.Tensor] = None,
                        ref: Optional[torch.Tensor] = None, mismatches: Optional[torch.Tensor] = None,
                        lut: Optional[torch.Tensor] = None, gains: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Spec decode of packed bytes (a uint8 CUDA tensor, 64-byte aligned) into out [R, K] fp32 (allocated when None
    and no ref is given); with ref, adds the number of positions whose value differs from ref to mismatches (int64
    CUDA tensor [1])."""
    _check_fmt(f)
    dev = data.device
    if lut is None or gains is None:
        lt, gt = _tables(f, dev)
        lut = lt if lut is None else lut
        gains = gt if gains is None else gains
    if out is None and ref is None:
        out = torch.empty((R, K), dtype=torch.float32, device=dev)
    masks = (ctypes.c_int * 3)(*([int(m) for m in f.masks] + [0, 0, 0])[:3])
    rc = _lib.lib().ltq_decode_slice(ptr(data), R, K, f.K, f.frac, f.h, f.sub, ctypes.cast(masks, ctypes.c_void_p),
                                     len(f.masks), ptr(lut), ptr(gains), ptr(out), out.stride(0) if out is not None else 0,
                                     ptr(ref), ref.stride(0) if ref is not None else 0, ptr(mismatches),
                                     _lib.stream_ptr(dev))
    if rc != 0:
        raise RuntimeError(f"ltq_decode_slice: error code {rc}")
    return out


def decode_slice(data, R: int, K: int, f: LtqFormat, device) -> torch.Tensor:
    """src/ltq_file.py:119-148: unscaled slice values [R, K] gain[g] * lut[label * U + u] per the spec."""
    dev = torch.device(device)
    if isinstance(data, torch.Tensor) and data.is_cuda:
        buf = data
    else:
        raw = np.frombuffer(bytes(data[: slice_bytes(R, K, f)]), dtype=np.uint8)
        buf = torch.empty(_align(max(raw.size, 1), 64), dtype=torch.uint8, device=dev)
        buf[: raw.size].copy_(torch.from_numpy(raw.copy()))
    return decode_slice_device(buf, R, K, f)


def fwht_inplace(x: torch.Tensor, block_size: int = TILE) -> torch.Tensor:
    from .liqk_v2 import fwht_inplace as fw
    return fw(x, block_size)


def assemble(G: torch.Tensor, d_row: torch.Tensor, e: torch.Tensor, suh: torch.Tensor) -> torch.Tensor:
    """W = H256(d q) * suh over columns, d[m, b] = d_row[m] 2^(e[m, b] / 4) (src/ltq_file.py:151-156)."""
    M, K = G.shape
    scale = d_row.float().unsqueeze(1) * torch.exp2(0.25 * e.float())
    W = (scale.unsqueeze(2) * G.view(M, K // TILE, TILE)).view(M, K)
    return fwht_inplace(W, block_size=TILE) * suh.float().unsqueeze(0)


def rotate_input(x: torch.Tensor, suh: torch.Tensor) -> torch.Tensor:
    """x_rot = H256(suh * x) for x [..., K]: the input of the packed-matrix product (W x = (d val) x_rot for
    W = H256(d val) * suh, the block FWHT being symmetric)."""
    from .liqk_v2 import fwht_rows_scaled
    K = x.shape[-1]
    return fwht_rows_scaled(x.reshape(-1, K).float().contiguous(), suh.float().contiguous(), mode=2).reshape(x.shape)


def matvec_slice_device(data: torch.Tensor, R: int, K: int, f: LtqFormat, d_row: torch.Tensor, e: torch.Tensor,
                        x_rot: torch.Tensor, y: Optional[torch.Tensor] = None, lut: Optional[torch.Tensor] = None,
                        gains: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y [R] = (d val) x_rot for one packed slice (ltq_matvec_slice): val the spec-decoded tile values, d = d_row (fp16
    [R]) * 2^(e [R, K/256] / 4), x_rot = rotate_input(x, suh) [K] fp32."""
    _check_fmt(f)
    dev = data.device
    if lut is None or gains is None:
        lt, gt = _tables(f, dev)
        lut = lt if lut is None else lut
        gains = gt if gains is None else gains
    if y is None:
        y = torch.empty(R, dtype=torch.float32, device=dev)
    dh = d_row.to(torch.float16).contiguous()
    ec = e.to(torch.int8).contiguous()
    xr = x_rot.float().contiguous()
    masks = (ctypes.c_int * 3)(*([int(m) for m in f.masks] + [0, 0, 0])[:3])
    rc = _lib.lib().ltq_matvec_slice(ptr(data), R, K, f.K, f.frac, f.h, f.sub, ctypes.cast(masks, ctypes.c_void_p),
                                     len(f.masks), ptr(lut), ptr(gains), ptr(dh), ptr(ec), ec.stride(0), ptr(xr),
                                     ptr(y), _lib.stream_ptr(dev))
    if rc != 0:
        raise RuntimeError(f"ltq_matvec_slice: error code {rc}")
    return y


def matvec(data: torch.Tensor, slices, formats: List[LtqFormat], d_row: torch.Tensor, e: torch.Tensor,
           suh: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """y = W x [M] for a packed matrix (its .ltq data tensor on the device, 64-byte aligned, and the slice table rows
    [r0, r1, format, offset]) without decoding it to memory: one input rotation, one kernel per row slice."""
    K = suh.shape[0]
    M = d_row.shape[0]
    xr = rotate_input(x.reshape(K).to(data.device), suh.to(data.device))
    y = torch.empty(M, dtype=torch.float32, device=data.device)
    for r0, r1, fi, off in (slices.tolist() if torch.is_tensor(slices) else slices):
        matvec_slice_device(data[off:], r1 - r0, K, formats[fi], d_row[r0:r1].to(data.device),
                            e[r0:r1].to(data.device), xr, y=y[r0:r1])
    return y


def pack_matrix_device(m: dict, formats: Dict[str, LtqFormat], verify: bool = True):
    """All row slices of a quantized matrix (liqk_v2.PACK["matrix"] fields, device tensors) packed into one uint8 CUDA
    buffer laid out as the .ltq data tensor (each slice at a multiple of 64 bytes), and the slice table rows
    [r0, r1, format, offset] (format = position in `formats`).  With verify, returns also an int64 [1] CUDA tensor: the
    number of weights whose spec decode differs from the quantizer's tile values (0 when the file is right)."""
    M, K = m["idx"].shape
    names = list(formats)
    rows, off = [], 0
    for r0, r1, sp in m["row_slices"]:
        off = _align(off, 64)
        rows.append([r0, r1, names.index(sp), off])
        off += slice_bytes(r1 - r0, K, formats[sp])
    dev = m["idx"].device
    buf = torch.zeros(_align(max(off, 1), 64), dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int64, device=dev) if verify else None
    for (r0, r1, fi, o), (_, _, sp) in zip(rows, m["row_slices"]):
        f = formats[sp]
        n = slice_bytes(r1 - r0, K, f)
        seg = buf[o: o + _align(max(n, 1), 64)]
        pack_slice_device(m["idx"][r0:r1], m["gi"][r0:r1], f, out=seg)
        if verify:
            G = m["G"][r0:r1]
            decode_slice_device(seg, r1 - r0, K, f, ref=G if G.stride(1) == 1 else G.contiguous(), mismatches=bad)
    return buf[:off], rows, bad


class LtqWriter:
    """Writes data straight to the file: `reserve` bytes are reserved for the header (data starts at 16 + reserve, a
    multiple of 4096); `finalize` writes the header, space-padded to the same length (src/ltq_file.py:163-223)."""

    def __init__(self, path: Path, formats: List[LtqFormat], reserve: int = (64 << 20) - 16):
        assert (16 + reserve) % 4096 == 0
        self.path, self.reserve = Path(path), reserve
        self.formats = formats
        self.fmt_index = {f.name: i for i, f in enumerate(formats)}
        self.f = open(self.path, "wb")
        self.f.write(bytes(16 + reserve))
        self.cur = 0
        self.tensors = {}
        self.quantized = []

    def _write(self, name: str, raw: bytes, dtype: str, shape: list, align: int = 64):
        pad = _align(self.cur, align) - self.cur
        if pad:
            self.f.write(bytes(pad))
            self.cur += pad
        self.tensors[name] = {"dtype": dtype, "shape": [int(s) for s in shape], "offset": self.cur}
        self.f.write(raw)
        self.cur += len(raw)

    def add_tensor(self, name: str, t: torch.Tensor):
        t = t.detach().cpu().contiguous()
        dt = TORCH_TO_LTQ[t.dtype]
        raw = t.view(torch.int16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
        self._write(name, raw, dt, list(t.shape))

    def add_matrix(self, p: str, m: dict, verify: bool = True) -> int:
        """Matrix from liqk_v2.PACK["matrix"]; returns the byte size of its fields.  verify: the spec decode of each
        slice from the packed bytes must match the quantizer's tile values bit for bit (checked on the device)."""
        M, K = m["idx"].shape
        fmts = {f.name: f for f in self.formats}
        used = {sp: fmts[sp] for _, _, sp in m["row_slices"]}
        data, rows, bad = pack_matrix_device(m, used, verify)
        if verify and int(bad.item()):
            raise RuntimeError(f"{p}: decode disagrees with the quantizer in {int(bad.item())} weights")
        rows = [[r0, r1, self.fmt_index[list(used)[fi]], o] for r0, r1, fi, o in rows]
        self.add_tensor(f"{p}.ltq.slices", torch.tensor(rows, dtype=torch.int32))
        self._write(f"{p}.ltq.data", data.cpu().numpy().tobytes(), "u8", [int(data.numel())])
        self.add_tensor(f"{p}.ltq.d_row", m["d_row"].to(torch.float16))
        self.add_tensor(f"{p}.ltq.e", m["e"].to(torch.int8))
        self.add_tensor(f"{p}.ltq.suh", m["suh"].to(torch.float16))
        self.quantized.append(p)
        return int(data.numel()) + 16 * len(rows) + 2 * M + M * (K // TILE) + 2 * K

    def finalize(self, header: dict):
        header = dict(header, tensors=self.tensors)
        raw = json.dumps(header, ensure_ascii=False, separators=(",", ":")).encode("utf-8")
        assert len(raw) <= self.reserve, f"header of {len(raw)} B does not fit in the {self.reserve} B reserve"
        self.f.seek(0)
        self.f.write(MAGIC + struct.pack("<IQ", VERSION, self.reserve) + raw + b" " * (self.reserve - len(raw)))
        self.f.close()


class LtqFile:
    """Reader (src/ltq_file.py:245-277)."""

    def __init__(self, path: Path):
        with open(path, "rb") as f:
            magic, (ver, H) = f.read(4), struct.unpack("<IQ", f.read(12))
            assert magic == MAGIC and ver == VERSION, (magic, ver)
            self.header = json.loads(f.read(H).decode("utf-8"))
        self.data_off = 16 + H
        assert self.data_off % 4096 == 0
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.formats = [format_from_json(d) for d in self.header["quantization"]["formats"]]

    def raw(self, name: str) -> memoryview:
        t = self.header["tensors"][name]
        n = int(np.prod(t["shape"])) * np.dtype(DTYPES[t["dtype"]][0]).itemsize
        o = self.data_off + t["offset"]
        return memoryview(self.mm[o: o + n])

    def tensor(self, name: str) -> torch.Tensor:
        t = self.header["tensors"][name]
        np_dt, th_dt = DTYPES[t["dtype"]]
        arr = torch.from_numpy(np.frombuffer(self.raw(name), dtype=np_dt).copy()).reshape(t["shape"])
        return arr.view(torch.bfloat16) if t["dtype"] == "bf16" else arr

    def decode_matrix(self, p: str, device="cuda") -> torch.Tensor:
        """Matrix W [M, K] float32, as reconstructed by the engine (spec decode on the device)."""
        d_row, e, suh = (self.tensor(f"{p}.ltq.{k}").to(device) for k in ("d_row", "e", "suh"))
        M, K = d_row.shape[0], suh.shape[0]
        raw = np.frombuffer(self.raw(f"{p}.ltq.data"), dtype=np.uint8)
        data = torch.empty(_align(max(raw.size, 1), 64), dtype=torch.uint8, device=device)
        data[: raw.size].copy_(torch.from_numpy(raw.copy()))
        G = torch.empty((M, K), device=device)
        for r0, r1, fi, off in self.tensor(f"{p}.ltq.slices").tolist():
            decode_slice_device(data[off:], r1 - r0, K, self.formats[fi], out=G[r0:r1])
        return assemble(G, d_row, e, suh)

    def matvec(self, p: str, x: torch.Tensor, device="cuda") -> torch.Tensor:
        """y = W x for matrix p, computed from its packed tiles on the device (ltq_matvec_slice)."""
        d_row, e, suh = (self.tensor(f"{p}.ltq.{k}").to(device) for k in ("d_row", "e", "suh"))
        raw = np.frombuffer(self.raw(f"{p}.ltq.data"), dtype=np.uint8)
        data = torch.empty(_align(max(raw.size, 1), 64), dtype=torch.uint8, device=device)
        data[: raw.size].copy_(torch.from_numpy(raw.copy()))
        return matvec(data, self.tensor(f"{p}.ltq.slices"), self.formats, d_row, e, suh, x)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--check", type=Path, required=True)
    ap.add_argument("--n", type=int, default=4, help="how many matrices to decode in full")
    args = ap.parse_args()
    lf = LtqFile(args.check)
    q = lf.header["quantization"]
    print(f"{args.check}: {args.check.stat().st_size / 1e9:.2f} GB, tensors {len(lf.header['tensors'])}, formats "
          f"{len(q['formats'])}, bits/weight {q.get('bits_per_weight')}")
    names = sorted({k[: -len(".ltq.data")] for k in lf.header["tensors"] if k.endswith(".ltq.data")})
    for p in names[:: max(1, len(names) // args.n)][: args.n]:
        W = lf.decode_matrix(p)
        print(f"{p}: {tuple(W.shape)}, rms {W.square().mean().sqrt():.4g}, finite {bool(torch.isfinite(W).all())}")


if __name__ == "__main__":
    main()
