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
import os
import struct
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import ptr
from .formats import TILE, LtqFormat

# File layout (the .ltq container read by the reference and by lumen-format):
#   bytes 0..3   b"LTQ\0"
#   bytes 4..7   u32 container version (1), little endian
#   bytes 8..15  u64 H = length of the JSON header area, little endian
#   16 .. 16+H   UTF-8 JSON header, space-padded to H bytes; its "tensors" maps a name to {dtype, shape, offset}
#   16+H ..      data area (16 + H is a multiple of 4096); each tensor starts at a multiple of 64 bytes of it
MAGIC = b"LTQ\0"
VERSION = 1
DATA_ALIGN = 64
PAGE = 4096
# element type names of the header and their torch types (the container's dtype vocabulary)
LTQ_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "i32": torch.int32,
              "i8": torch.int8, "u8": torch.uint8}
_DTYPE_NAME = {v: k for k, v in LTQ_DTYPES.items()}
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


def _host_bytes(t: torch.Tensor) -> np.ndarray:
    """The little-endian bytes of a tensor's elements in row-major order, as a uint8 host array (any element type,
    bf16 included: the tensor is reinterpreted, not converted)."""
    t = t.detach()
    if t.dtype not in _DTYPE_NAME:
        raise TypeError(f"no .ltq element type for {t.dtype}")
    return t.contiguous().reshape(-1).view(torch.uint8).cpu().numpy()


class LtqWriter:
    """Streams an .ltq container to `path`.

    The first 16 + `reserve` bytes are the preamble and the header area, filled in by `finalize` (the header JSON is
    only complete once every tensor is placed); tensors go to the data area as they arrive, each at the next multiple
    of 64 bytes, by positioned writes (the gaps are file holes and read as zeros).  `add_matrix` takes a quantized
    matrix (liqk_v2.PACK["matrix"] fields on the device), packs its row slices on the device and checks them there
    before any byte is written.  Usable as a context manager; leaving the block without `finalize` closes the file
    with the header area still blank."""

    def __init__(self, path: Path, formats: List[LtqFormat], reserve: int = (64 << 20) - 16):
        if (16 + reserve) % PAGE:
            raise ValueError(f"reserve + 16 must be a multiple of {PAGE} (the data area starts on a page)")
        self.path = Path(path)
        self.reserve = int(reserve)
        self.formats = list(formats)
        self.fmt_index = {f.name: k for k, f in enumerate(self.formats)}
        self.tensors: Dict[str, dict] = {}
        self.quantized: List[str] = []
        self._data_start = 16 + self.reserve
        self._end = 0  # bytes of the data area used so far
        self._fd = os.open(self.path, os.O_RDWR | os.O_CREAT | os.O_TRUNC, 0o644)
        os.ftruncate(self._fd, self._data_start)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self):
        if self._fd is not None:
            os.close(self._fd)
            self._fd = None

    def _put(self, name: str, payload: np.ndarray, dtype: str, shape) -> int:
        """Places `payload` (uint8) at the next aligned offset of the data area and records it; returns the offset."""
        if name in self.tensors:
            raise KeyError(f"tensor {name} written twice")
        off = _align(self._end, DATA_ALIGN)
        view = memoryview(np.ascontiguousarray(payload, dtype=np.uint8))
        done = 0
        while done < len(view):
            done += os.pwrite(self._fd, view[done:], self._data_start + off + done)
        self._end = off + len(view)
        self.tensors[name] = {"dtype": dtype, "shape": [int(d) for d in shape], "offset": off}
        return off

    def add_tensor(self, name: str, t: torch.Tensor):
        """A plain tensor (f32 / f16 / bf16 / i32 / i8 / u8), copied to the host as its raw element bytes."""
        self._put(name, _host_bytes(t), _DTYPE_NAME[t.dtype], tuple(t.shape))

    def add_matrix(self, p: str, m: dict, verify: bool = True) -> int:
        """The five tensors of quantized matrix `p` (`{p}.ltq.slices` [n, 4] i32 rows [r0, r1, format, offset],
        `.data` the packed slices, `.d_row` f16, `.e` i8, `.suh` f16); returns their total bytes.  With verify the spec
        decode of every packed slice must reproduce the quantizer's tile values bit for bit (checked on the device)."""
        M, K = m["idx"].shape
        used: Dict[str, LtqFormat] = {}
        for _, _, spec in m["row_slices"]:
            if spec not in self.fmt_index:
                raise KeyError(f"{p}: format {spec} is not among the writer's formats")
            used.setdefault(spec, self.formats[self.fmt_index[spec]])
        data, rows, bad = pack_matrix_device(m, used, verify)
        if verify:
            n_bad = int(bad.item())
            if n_bad:
                raise RuntimeError(f"{p}: decode disagrees with the quantizer in {n_bad} weights")
        local = list(used)
        table = torch.tensor([[r0, r1, self.fmt_index[local[fi]], o] for r0, r1, fi, o in rows], dtype=torch.int32)
        fields = [("slices", table), ("data", data), ("d_row", m["d_row"].to(torch.float16)),
                  ("e", m["e"].to(torch.int8)), ("suh", m["suh"].to(torch.float16))]
        total = 0
        for key, t in fields:
            self.add_tensor(f"{p}.ltq.{key}", t)
            total += t.numel() * t.element_size()
        self.quantized.append(p)
        return total

    def finalize(self, header: dict):
        """Writes the preamble and the header (the caller's fields plus "tensors") and closes the file."""
        blob = json.dumps(dict(header, tensors=self.tensors), ensure_ascii=False, separators=(",", ":")).encode("utf-8")
        if len(blob) > self.reserve:
            raise ValueError(f"header of {len(blob)} bytes does not fit the {self.reserve}-byte header area")
        pre = MAGIC + struct.pack("<IQ", VERSION, self.reserve)
        os.pwrite(self._fd, pre + blob.ljust(self.reserve, b" "), 0)
        self.close()


class LtqFile:
    """Read access to an .ltq container: the header, each tensor's bytes (memory-mapped), tensors, and the quantized
    matrices decoded (or multiplied with a vector) on the device from their packed tiles."""

    def __init__(self, path: Path):
        self.path = Path(path)
        with open(self.path, "rb") as fh:
            pre = fh.read(16)
            if len(pre) < 16 or pre[:4] != MAGIC:
                raise ValueError(f"{self.path}: not an .ltq file")
            version, hlen = struct.unpack("<IQ", pre[4:])
            if version != VERSION:
                raise ValueError(f"{self.path}: container version {version}, expected {VERSION}")
            self.header = json.loads(fh.read(hlen).decode("utf-8"))
        self.data_off = 16 + hlen
        if self.data_off % PAGE:
            raise ValueError(f"{self.path}: the data area starts at {self.data_off}, not on a {PAGE}-byte page")
        self.mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        self.formats = [format_from_json(d) for d in self.header["quantization"]["formats"]]

    def _entry(self, name: str):
        e = self.header["tensors"][name]
        dt = LTQ_DTYPES[e["dtype"]]
        count = 1
        for d in e["shape"]:
            count *= int(d)
        return e, dt, count * torch.empty((), dtype=dt).element_size()

    def raw(self, name: str) -> memoryview:
        """The tensor's bytes in the file (no copy)."""
        e, _, nbytes = self._entry(name)
        o = self.data_off + e["offset"]
        return memoryview(self.mm[o: o + nbytes])

    def tensor(self, name: str) -> torch.Tensor:
        """The tensor as a host torch tensor of its stored element type and shape."""
        e, dt, nbytes = self._entry(name)
        if nbytes == 0:
            return torch.empty(e["shape"], dtype=dt)
        return torch.frombuffer(bytearray(self.raw(name)), dtype=dt).reshape(e["shape"])

    def matrices(self) -> List[str]:
        """Names of the quantized matrices in the file, in data order."""
        tail = ".ltq.data"
        found = [(e["offset"], k[: -len(tail)]) for k, e in self.header["tensors"].items() if k.endswith(tail)]
        return [k for _, k in sorted(found)]

    def _device_fields(self, p: str, device):
        d_row, e, suh = (self.tensor(f"{p}.ltq.{k}").to(device) for k in ("d_row", "e", "suh"))
        raw = self.tensor(f"{p}.ltq.data")
        data = torch.zeros(_align(max(raw.numel(), 1), DATA_ALIGN), dtype=torch.uint8, device=device)
        data[: raw.numel()].copy_(raw)
        return data, self.tensor(f"{p}.ltq.slices").tolist(), d_row, e, suh

    def decode_matrix(self, p: str, device="cuda") -> torch.Tensor:
        """Matrix `p` [M, K] fp32 as an inference engine rebuilds it: spec decode of every slice on the device, block
        scales, inverse rotation, column scales."""
        data, slices, d_row, e, suh = self._device_fields(p, device)
        M, K = d_row.shape[0], suh.shape[0]
        G = torch.empty((M, K), device=device)
        for r0, r1, fi, off in slices:
            decode_slice_device(data[off:], r1 - r0, K, self.formats[fi], out=G[r0:r1])
        return assemble(G, d_row, e, suh)

    def matvec(self, p: str, x: torch.Tensor, device="cuda") -> torch.Tensor:
        """y = W x for matrix p, computed from its packed tiles on the device (ltq_matvec_slice)."""
        data, slices, d_row, e, suh = self._device_fields(p, device)
        return matvec(data, slices, self.formats, d_row, e, suh, x)


def main(argv=None):
    """`--check FILE`: reads the container, lists its size and formats, and rebuilds a spread of its matrices on the
    device (finite values, RMS)."""
    ap = argparse.ArgumentParser(description="inspect an .ltq file")
    ap.add_argument("--check", type=Path, required=True)
    ap.add_argument("--n", type=int, default=4, help="number of matrices to rebuild")
    a = ap.parse_args(argv)
    lf = LtqFile(a.check)
    quant = lf.header["quantization"]
    names = lf.matrices()
    size_gb = a.check.stat().st_size / 1e9
    print(f"{a.check}: {size_gb:.2f} GB; {len(lf.header['tensors'])} tensors, {len(names)} quantized matrices; formats "
          f"{', '.join(f.name for f in lf.formats)}; bits/weight {quant.get('bits_per_weight')}")
    step = max(1, len(names) // max(a.n, 1))
    for p in names[::step][: a.n]:
        W = lf.decode_matrix(p)
        rms = float(W.double().square().mean().sqrt())
        print(f"  {p}: {list(W.shape)}  rms {rms:.4g}  all finite: {bool(torch.isfinite(W).all())}")


if __name__ == "__main__":
    main()
