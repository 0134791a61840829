"""Weight-format converter: a native `weights.bin` + `index.json` in any matrix kind to the same
model in another kind.

The input is what `scripts/convert_weights.py` of the reference writes (block-32 "q4" matrices,
the kind assumed when an entry has none) or a file in the "f16" / "q4g64" kinds this engine adds.
The output keeps that file's conventions (scripts/convert_weights.py:35-54): every tensor starts
on a 256-byte boundary, and byte-identical tensors of the same kind are stored once (the tied
embedding / LM head). Non-matrix tensors (norm weights, conv weights, GDN parameters) are copied.

Kinds (value(r, c) as the kernels decode it, kernels/src/lib.rs:141-155,484-497 for "q4"):
  f16    w f16[rows][k]
  q4     w u4[rows][k] packed 8 per u32, low nibble first; s f16[rows][k/32] (two per u32, even
         block in the low half); z u4[rows][k/32] packed 8 per u32; value = (q - z) * s
  q4g64  w as q4; s f16[rows][k/64]; z f16[rows][k/64]; value = (q - z) * s

Conversions: a matrix already in the target kind is copied byte for byte. Otherwise it is decoded
to f32 with the kernels' arithmetic ((float(q) - z) * s, one rounding per operation) and encoded:
  * to f16 by round-to-nearest-even (so q4 -> f16 is exact up to one f16 rounding per value);
  * to q4 / q4g64 by asymmetric min-max 4-bit quantization per group (32 / 64 values along k):
    the group's range [min(x, 0), max(x, 0)] is split into 15 steps, s = f16(range / 15),
    z = -min / s (rounded to an integer in 0..15 for q4, whose zero points are nibbles; kept as
    f16 for q4g64), q = clamp(rint(x / s + z), 0, 15). Every value decodes to within about half
    a step (s / 2) of the input.
Requantizing int4 to another int4 grouping loses precision; converting from f16 is the intended
use of the int4 targets.

Usage: python -m qne.convert SRC_DIR OUT_DIR --kind f16|q4|q4g64 [--embed-kind KIND]
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import os
from pathlib import Path

import numpy as np

ALIGN = 256
KINDS = ("f16", "q4", "q4g64")
_PARTS = {"f16": ("w",), "q4": ("w", "s", "z"), "q4g64": ("w", "s", "z")}
_GROUP = {"q4": 32, "q4g64": 64}


def part_bytes(kind: str, rows: int, k: int) -> dict:
    """Byte size of each part of a rows x k matrix of `kind` (the loader's size check)."""
    el = rows * k
    if kind == "f16":
        return {"w": el * 2}
    if kind == "q4":
        return {"w": el // 2, "s": el // 16, "z": el // 64}
    if kind == "q4g64":
        return {"w": el // 2, "s": el // 32, "z": el // 32}
    raise ValueError(f"unknown matrix kind {kind!r}")


def decode_rows(kind: str, parts: dict, rows: int, k: int, r0: int, r1: int) -> np.ndarray:
    """Rows r0..r1 of a matrix as f32, with the kernels' arithmetic."""
    n = r1 - r0
    if kind == "f16":
        return parts["w"].view(np.float16).reshape(rows, k)[r0:r1].astype(np.float32)
    g = _GROUP[kind]
    wb = parts["w"].view(np.uint8).reshape(rows, k // 2)[r0:r1]
    q = np.empty((n, k), np.float32)
    q[:, 0::2] = wb & 15
    q[:, 1::2] = wb >> 4
    s = parts["s"].view(np.float16).reshape(rows, k // g)[r0:r1].astype(np.float32)
    if kind == "q4":
        zb = parts["z"].view(np.uint8).reshape(rows, k // 64)[r0:r1]
        z = np.empty((n, k // 32), np.float32)
        z[:, 0::2] = zb & 15
        z[:, 1::2] = zb >> 4
    else:
        z = parts["z"].view(np.float16).reshape(rows, k // g)[r0:r1].astype(np.float32)
    out = (q.reshape(n, k // g, g) - z[..., None]) * s[..., None]
    return out.reshape(n, k)


def encode_rows(kind: str, x: np.ndarray) -> dict:
    """f32 rows [n][k] -> the parts of `kind` for those rows (bytes in file order)."""
    n, k = x.shape
    if kind == "f16":
        return {"w": x.astype(np.float16)}
    g = _GROUP[kind]
    xb = x.reshape(n, k // g, g)
    lo = np.minimum(xb.min(axis=-1), 0.0)
    hi = np.maximum(xb.max(axis=-1), 0.0)
    with np.errstate(over="ignore"):
        s_h = ((hi - lo) / np.float32(15)).astype(np.float16)
    if not np.all(np.isfinite(s_h)):
        raise ValueError("a group's range does not fit an f16 scale")
    s = s_h.astype(np.float32)
    div = np.where(s > 0, s, np.float32(1))
    z = -lo / div
    if kind == "q4":
        z = np.clip(np.rint(z), 0, 15)
    z_h = z.astype(np.float16)
    zf = z_h.astype(np.float32)
    q = np.clip(np.rint(xb / div[..., None] + zf[..., None]), 0, 15).astype(np.uint8).reshape(n, k)
    out = {"w": (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8), "s": s_h}
    if kind == "q4":
        zi = zf.astype(np.uint8)
        out["z"] = (zi[:, 0::2] | (zi[:, 1::2] << 4)).astype(np.uint8)
    else:
        out["z"] = z_h
    return out


class _Writer:
    """Appends tensors 256-byte aligned; byte-identical tensors of one kind are stored once."""

    def __init__(self, f):
        self.f = f
        self.offset = 0
        self.index = {}
        self.content = {}

    def add(self, name: str, chunks, kind: str) -> None:
        h = hashlib.sha256()
        data = [np.ascontiguousarray(c).view(np.uint8).ravel() for c in chunks]
        for d in data:
            h.update(d.data)
        key = (kind, sum(d.size for d in data), h.digest())
        if key in self.content:
            self.index[name] = dict(self.content[key])
            return
        pad = (-self.offset) % ALIGN
        self.f.write(b"\0" * pad)
        self.offset += pad
        entry = {"offset": self.offset, "bytes": int(key[1]), "kind": kind}
        for d in data:
            self.f.write(d.data)
        self.offset += key[1]
        self.index[name] = entry
        self.content[key] = entry


def _source_parts(index: dict, weights: np.ndarray, name: str, kind: str, rows: int, k: int) -> dict:
    parts = {}
    for part, nbytes in part_bytes(kind, rows, k).items():
        t = index["tensors"].get(f"{name}.{part}")
        if t is None or int(t["bytes"]) != nbytes:
            raise ValueError(f"invalid tensor size: {name}.{part}")
        off = int(t["offset"])
        if off + nbytes > weights.size:
            raise ValueError(f"invalid tensor range: {name}.{part}")
        parts[part] = weights[off:off + nbytes]
    return parts


def _part_kind(kind: str, part: str) -> str:
    if kind == "f16" or part == "w":
        return kind
    return "u8" if (kind == "q4" and part == "z") else "f16"  # the reference's kind names


def convert_to(index_json: str, weights, out, kind: str, embed_kind: str | None = None,
               chunk_elems: int = 1 << 24) -> dict:
    """Writes the converted weights to the binary file object `out`; returns the new index.

    `kind` applies to the decoder matrices, `embed_kind` (default `kind`) to embed and lm_head."""
    if kind not in KINDS or (embed_kind is not None and embed_kind not in KINDS):
        raise ValueError(f"kind must be one of {KINDS}")
    embed_kind = embed_kind or kind
    index = json.loads(index_json)
    w = np.asarray(weights).view(np.uint8).ravel()
    wr = _Writer(out)
    matrices = {}
    parts_of = set()
    done = {}  # (source part ranges, target kind) -> output index entries
    for name, spec in index["matrices"].items():
        rows, k = int(spec["rows"]), int(spec["k"])
        src_kind = spec.get("kind", "q4")
        dst_kind = embed_kind if name in ("embed", "lm_head") else kind
        if src_kind not in KINDS:
            raise ValueError(f"{name}: unknown matrix kind {src_kind!r}")
        if dst_kind != "f16" and k % 64:
            raise ValueError(f"{name}: int4 kinds need k % 64 == 0 (k = {k})")
        src = _source_parts(index, w, name, src_kind, rows, k)
        parts_of.update(f"{name}.{p}" for p in src)
        key = (tuple((p, int(index["tensors"][f"{name}.{p}"]["offset"])) for p in sorted(src)), src_kind, dst_kind)
        matrices[name] = {"rows": rows, "k": k, "kind": dst_kind}
        if key in done:  # the same source tensors (a tied LM head): same output
            for p, e in done[key].items():
                wr.index[f"{name}.{p}"] = dict(e)
            continue
        if src_kind == dst_kind:
            outs = {p: [src[p]] for p in src}
        else:
            step = max(1, chunk_elems // k)
            outs = {p: [] for p in _PARTS[dst_kind]}
            for r0 in range(0, rows, step):
                enc = encode_rows(dst_kind, decode_rows(src_kind, src, rows, k, r0, min(rows, r0 + step)))
                for p in outs:
                    outs[p].append(enc[p])
        for p in _PARTS[dst_kind]:
            wr.add(f"{name}.{p}", outs[p], _part_kind(dst_kind, p))
        done[key] = {p: wr.index[f"{name}.{p}"] for p in _PARTS[dst_kind]}
    for name, t in index["tensors"].items():
        if name in parts_of:
            continue
        off, nbytes = int(t["offset"]), int(t["bytes"])
        if off + nbytes > w.size:
            raise ValueError(f"invalid tensor range: {name}")
        wr.add(name, [w[off:off + nbytes]], t.get("kind", "f32"))
    new = {k_: v for k_, v in index.items() if k_ not in ("matrices", "tensors")}
    new["source"] = f"{index.get('source', 'unknown')}, converted to {kind}" + (
        f" (embed/lm_head {embed_kind})" if embed_kind != kind else "")
    new["format_version"] = 1
    new["matrices"] = matrices
    new["tensors"] = wr.index
    return new


def convert(index_json: str, weights, kind: str, embed_kind: str | None = None) -> tuple[str, np.ndarray]:
    """In memory: (index.json text, weights as uint8) of the converted model."""
    buf = io.BytesIO()
    new = convert_to(index_json, weights, buf, kind, embed_kind)
    return json.dumps(new, indent=1), np.frombuffer(buf.getbuffer(), np.uint8).copy()


def convert_dir(src: Path, dst: Path, kind: str, embed_kind: str | None = None) -> dict:
    """SRC/{index.json, weights.bin} -> DST/{index.json, weights.bin}; files appear whole or not at all."""
    src, dst = Path(src), Path(dst)
    index_json = (src / "index.json").read_text(encoding="utf-8")
    weights = np.memmap(src / "weights.bin", dtype=np.uint8, mode="r")
    dst.mkdir(parents=True, exist_ok=True)
    tmp_w, tmp_i = dst / "weights.bin.tmp", dst / "index.json.tmp"
    with open(tmp_w, "wb") as f:
        new = convert_to(index_json, weights, f, kind, embed_kind)
    tmp_i.write_text(json.dumps(new, indent=1), encoding="utf-8")
    os.replace(tmp_w, dst / "weights.bin")
    os.replace(tmp_i, dst / "index.json")
    return new


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Convert a native weights.bin + index.json to another matrix kind")
    ap.add_argument("src", type=Path, help="directory holding index.json and weights.bin")
    ap.add_argument("dst", type=Path, help="output directory")
    ap.add_argument("--kind", required=True, choices=KINDS, help="kind of the decoder matrices")
    ap.add_argument("--embed-kind", choices=KINDS, help="kind of embed and lm_head (default: --kind)")
    args = ap.parse_args(argv)
    new = convert_dir(args.src, args.dst, args.kind, args.embed_kind)
    total = max(int(t["offset"]) + int(t["bytes"]) for t in new["tensors"].values())
    print(f"wrote {total / 1e6:.0f} MB, {len(new['tensors'])} tensors to {args.dst}")


if __name__ == "__main__":
    main()
