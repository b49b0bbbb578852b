"""safetensors -> detwgt v2 converter (model ingestion for the det path).

Restates casettek/raster-inference ``tools/gemma-det-num-wgt-converter/
main.rs:218-560`` with ``src/shared/numerics/det_num/convert.rs:77-189``:

* the source is a model directory (``config.json`` plus ``model.safetensors``
  or ``consolidated.safetensors``) or a ``.safetensors`` file whose directory
  (or ``--config``) holds ``config.json``; the output directory must be new or
  empty, and receives ``model.detwgt`` and a copy of ``config.json``;
* tensors are written in byte-wise sorted name order;
* every F32 / BF16 / F16 value becomes a Q16.16 weight,
  ``sat_i32(round_ties_even(x * 65536))``; a non-finite value is an error.
  ``x * 65536`` is exact in float64 for every finite float32 (an exponent
  shift), and numpy's ``rint`` rounds half to even, so the vectorised form
  gives the reference's bit-level result for every input;
* the overflow bound: in a tensor of rank >= 2 every row (last dimension) must
  have mass ``sum |w|`` below 2^31, else the conversion fails naming the row;
  rank-1 tensors record their mass without the check;
* a tensor whose every value fits i16 is stored at half width.

Conversion is a one-time step per model, streamed tensor by tensor (memory
holds one tensor at a time): each tensor's rows convert in chunks on all host
cores, or with ``--device N`` on that GPU (``rdet_convert_to_wgt``, the same
results); the GPU loads the output.

    python -m raster-inference_b200.convert --input <model-dir-or-safetensors> \\
        --output-dir <new-dir> [--config config.json] [--device N] [--report-bounds] [--report-widths]
"""
from __future__ import annotations

import argparse
import json
import mmap
import os
import shutil
import struct
import sys
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import detwgt

ROW_MASS_LIMIT = 1 << 31  # DET_WGT_ROW_MASS_LIMIT (det_num/mod.rs:17)
_WIDTH = {"F32": 4, "BF16": 2, "F16": 2}


_F32_BELOW_2_31 = np.float32(2147483520.0)  # the largest float32 below 2^31


def f32_to_wgt_bits(x: np.ndarray) -> np.ndarray:
    """convert.rs:77-93 f32_to_wgt over an array: Q16.16 bits (int32).

    x * 65536 is exact in float32 (an exponent shift; a product beyond the
    float32 range becomes an infinity of the right sign, which saturates like
    the reference), ``rint`` rounds half to even, and every float32 below 2^31
    in magnitude is an integer the int32 cast keeps."""
    x = np.asarray(x, dtype=np.float32)
    if x.size and not np.isfinite(x).all():
        raise ValueError("f32_to_wgt requires a finite source value")
    with np.errstate(over="ignore"):
        y = np.rint(x * np.float32(65536.0))
    out = np.clip(y, np.float32(-2147483648.0), _F32_BELOW_2_31).astype(np.int32)
    out[y > _F32_BELOW_2_31] = 2147483647
    return out


def decode_values(raw, dtype: str) -> np.ndarray:
    """main.rs:544-550 decode_scalar for a whole little-endian buffer."""
    if dtype == "F32":
        return np.frombuffer(raw, dtype="<f4")
    if dtype == "F16":
        return np.frombuffer(raw, dtype="<f2").astype(np.float32)
    if dtype == "BF16":
        return (np.frombuffer(raw, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
    raise ValueError(f"unsupported tensor dtype {dtype}")


def _convert_rows(raw, dtype: str, row: int, r0: int, r1: int, out: np.ndarray, mass: np.ndarray):
    """Rows [r0, r1) of a tensor: Q16.16 bits into out, row masses into mass."""
    w = _WIDTH[dtype]
    bits = f32_to_wgt_bits(decode_values(raw[r0 * row * w:r1 * row * w], dtype))
    out[r0 * row:r1 * row] = bits
    # |INT32_MIN| wraps to itself in int32; as uint32 it is the magnitude 2^31
    mass[r0:r1] = np.abs(bits).view(np.uint32).reshape(-1, row).sum(axis=1, dtype=np.uint64)


def convert_tensor(raw, dtype: str, shape, pool=None, chunk_values: int = 1 << 22):
    """A whole tensor: (int32 bits, per-row masses), rows split across the
    worker pool in chunks of about ``chunk_values`` values."""
    n = int(np.prod(shape)) if len(shape) else 1
    row = max(int(shape[-1]) if len(shape) else 1, 1)
    rows = n // row if n else 0
    out = np.empty(n, dtype=np.int32)
    mass = np.zeros(rows, dtype=np.uint64)
    step = max(1, chunk_values // row)
    spans = [(r, min(rows, r + step)) for r in range(0, rows, step)]
    if pool is None or len(spans) < 2:
        for r0, r1 in spans:
            _convert_rows(raw, dtype, row, r0, r1, out, mass)
    else:
        for f in [pool.submit(_convert_rows, raw, dtype, row, r0, r1, out, mass) for r0, r1 in spans]:
            f.result()
    return out, mass


def convert_tensor_gpu(raw, dtype: str, shape, device: int):
    """convert_tensor on the GPU (rdet_convert_to_wgt): the raw values go to
    the device, the Q16.16 bits and row masses come back.  Same results as the
    host form; fails loudly when the CUDA library or device is missing."""
    import torch  # device memory only

    from . import convert_to_wgt

    n = int(np.prod(shape)) if len(shape) else 1
    row = max(int(shape[-1]) if len(shape) else 1, 1)
    rows = n // row if n else 0
    if n == 0:
        return np.empty(0, dtype=np.int32), np.zeros(0, dtype=np.uint64)
    dev = torch.device("cuda", device)
    src = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()).to(dev)
    out = torch.empty(n, dtype=torch.int32, device=dev)
    mass = torch.empty(rows, dtype=torch.int64, device=dev)
    stats = torch.zeros(2, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    convert_to_wgt(src.data_ptr(), dtype, rows, row, out.data_ptr(), mass.data_ptr(), stats.data_ptr(),
                   stream.cuda_stream)
    st = stats.cpu().numpy()
    if st[0]:
        raise ValueError("f32_to_wgt requires a finite source value")
    return out.cpu().numpy(), mass.cpu().numpy().view(np.uint64)


class SafeTensors:
    """A memory-mapped safetensors file: 8-byte LE header length, JSON header
    {name: {dtype, shape, data_offsets}}, then the data."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self._m = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._m[:8])
        if 8 + n > len(self._m):
            raise ValueError(f"{path}: header length {n} exceeds the file")
        header = json.loads(bytes(self._m[8:8 + n]))
        header.pop("__metadata__", None)
        self.base = 8 + n
        self.header = header

    def names(self):
        return sorted(self.header)  # sort_unstable on &str: byte order

    def tensor(self, name: str):
        h = self.header[name]
        b, e = h["data_offsets"]
        shape = tuple(int(d) for d in h["shape"])
        dtype = h["dtype"]
        if dtype not in _WIDTH:
            raise ValueError(f"tensor `{name}`: unsupported tensor dtype {dtype}")
        if e - b != int(np.prod(shape)) * _WIDTH[dtype]:
            raise ValueError(f"tensor `{name}`: {e - b} data bytes for shape {shape} of {dtype}")
        return dtype, shape, memoryview(self._m)[self.base + b:self.base + e]

    def close(self):
        try:
            self._m.close()
        except BufferError:  # a failed conversion's traceback still views the map
            pass
        self._f.close()


def write_safetensors(path: str, tensors) -> None:
    """Writes [(name, dtype, shape, bytes)] as a safetensors file (fixtures and
    tests; the format the converter reads)."""
    header, off, blobs = {}, 0, []
    for name, dtype, shape, data in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        off += len(data)
        blobs.append(data)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb)
        for data in blobs:
            f.write(data)


def _resolve(input_path: str, config: str | None):
    """main.rs:394-449 resolve_source."""
    if os.path.isdir(input_path):
        if config is not None:
            raise ValueError("--config is only supported when --input points to a `.safetensors` file")
        cfg = os.path.join(input_path, "config.json")
        if not os.path.isfile(cfg):
            raise ValueError(f"model directory {input_path} is missing config.json")
        for fn in ("model.safetensors", "consolidated.safetensors"):
            w = os.path.join(input_path, fn)
            if os.path.isfile(w):
                return w, cfg
        raise ValueError(f"model directory {input_path} is missing `model.safetensors` or `consolidated.safetensors`")
    if input_path.endswith(".safetensors"):
        cfg = config or os.path.join(os.path.dirname(input_path) or ".", "config.json")
        if not os.path.isfile(cfg):
            raise ValueError(f"could not locate config.json for {input_path}; pass --config explicitly")
        return input_path, cfg
    raise ValueError(f"unsupported input path {input_path}; expected a model directory or `.safetensors` file")


def _prepare_output(out: str):
    """main.rs:451-475 prepare_output_dir."""
    if os.path.exists(out):
        if not os.path.isdir(out):
            raise ValueError(f"output path {out} exists but is not a directory")
        if os.listdir(out):
            raise ValueError(f"output directory {out} must not already contain files")
    else:
        os.makedirs(out)


def _check_row_mass(name: str, shape, mass: np.ndarray) -> int:
    """main.rs:346-388 analyze_tensor: the max row mass; rows of rank >= 2
    tensors must stay below the limit."""
    if mass.size == 0:
        return 0
    if len(shape) >= 2:
        bad = np.nonzero(mass >= ROW_MASS_LIMIT)[0]
        if bad.size:
            r = int(bad[0])
            raise ValueError(f"tensor `{name}` failed the conversion-time overflow bound check: row {r} has row "
                             f"mass {int(mass[r])}, violating the overflow bound (must be < {ROW_MASS_LIMIT})")
    return int(mass.max())


def convert(input_path: str, output_dir: str, config: str | None = None, device: int | None = None) -> dict:
    """convert_model_to_det_num_wgt_artifact (main.rs:218-320): returns the
    summary (tensor count, input and output payload bytes, per-tensor width
    and max row mass).  device: a CUDA device ordinal converts the values on
    that GPU (rdet_convert_to_wgt), None on the host cores."""
    weights, cfg = _resolve(input_path, config)
    _prepare_output(output_dir)
    st = SafeTensors(weights)
    names = st.names()
    bounds = []
    in_bytes = out_bytes = 0

    def tensors():
        nonlocal in_bytes, out_bytes
        for name in names:
            dtype, shape, raw = st.tensor(name)
            in_bytes += len(raw)
            try:
                if device is None:
                    bits, row_mass = convert_tensor(raw, dtype, shape, pool)
                else:
                    bits, row_mass = convert_tensor_gpu(raw, dtype, shape, device)
            except ValueError as e:
                raise ValueError(f"failed to convert tensor `{name}` to Wgt: {e}") from None
            mass = _check_row_mass(name, shape, row_mass)
            width = 16 if (bits.size == 0 or (bits.min() >= -32768 and bits.max() <= 32767)) else 32
            out_bytes += bits.size * width // 8
            bounds.append({"name": name, "width": width, "max_row_mass": mass, "mac_bound": len(shape) >= 2,
                           "payload_bytes": bits.size * width // 8})
            yield name, shape, bits, mass

    out_w = os.path.join(output_dir, "model.detwgt")
    # numpy releases the GIL in these loops: row chunks convert on all cores
    pool = ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    try:
        with open(out_w, "wb") as f:
            detwgt.write(f, tensors(), len(names))
    finally:
        pool.shutdown()
        st.close()
    shutil.copyfile(cfg, os.path.join(output_dir, "config.json"))
    return {"tensor_count": len(names), "input_tensor_bytes": in_bytes, "output_tensor_bytes": out_bytes,
            "output_weights_path": out_w, "tensor_bounds": bounds}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="safetensors -> detwgt v2 (det_num Q16.16 weights)")
    ap.add_argument("--input", required=True)
    ap.add_argument("--output-dir", required=True)
    ap.add_argument("--config")
    ap.add_argument("--report-bounds", action="store_true")
    ap.add_argument("--report-widths", action="store_true")
    ap.add_argument("--device", type=int, default=None,
                    help="convert the values on this CUDA device (default: on the host cores)")
    a = ap.parse_args(argv)
    s = convert(a.input, a.output_dir, a.config, a.device)
    print(f"converted {s['tensor_count']} tensors: {s['input_tensor_bytes']} source bytes -> "
          f"{s['output_tensor_bytes']} payload bytes ({s['output_weights_path']})")
    b = s["tensor_bounds"]
    n16 = sum(1 for t in b if t["width"] == 16)
    by16 = sum(t["payload_bytes"] for t in b if t["width"] == 16)
    total = max(1, sum(t["payload_bytes"] for t in b))
    print(f"i16 width report: {n16}/{len(b)} tensors stored i16 ({100.0 * n16 / max(1, len(b)):.1f}% of tensors, "
          f"{100.0 * by16 / total:.1f}% of payload bytes)")
    if a.report_widths:
        print("Per-tensor storage widths:")
        for t in b:
            print(f"  {t['name']} width=i{t['width']} payload={t['payload_bytes']}")
    if a.report_bounds:
        print(f"Overflow-bound report (row mass limit = {ROW_MASS_LIMIT}):")
        for t in b:
            margin = "inf" if t["max_row_mass"] == 0 else f"{ROW_MASS_LIMIT / t['max_row_mass']:.2f}"
            note = "" if t["mac_bound"] else " (elementwise; not enforced)"
            print(f"  {t['name']} max_row_mass={t['max_row_mass']} margin={margin}x{note}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
