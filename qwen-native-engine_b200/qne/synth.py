"""Seeded synthetic Qwen3.5-shaped models in the reference's `weights.bin` + `index.json` format.

The format is the one `scripts/convert_weights.py` writes (tensors 256-byte aligned, tied
embedding / LM head stored once and referenced twice, projections concatenated: GDN mixer_in =
q, k, v, z, a, b; attention mixer_in = q, gate, k, v; gate_up = gate rows then up rows). Each
matrix entry carries a "kind": "f16", "q4" (the converter's MatMulNBits block-32 layout, the
default when absent) or "q4g64" (u4 packed 8 per u32, group 64 along k, f16 scale, f16 zero
point).

Values (benchmark configs): f16 weights N(0, std) rounded to f16; int4 weights uniform nibbles,
scales |N(0, scale_std)|, zero point 8; all norm weights 1; conv weights U(-0.5, 0.5);
GDN params dt_bias 0, A_neg_exp -0.5, norm 1 (the prototype's choices, kernels/src/lib.rs:773,777).
Every tensor draws from its own generator seeded by (seed, tensor index), so generation can run
in parallel and stays reproducible.
"""
from __future__ import annotations

import json
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ALIGN = 256
VOCAB = 248320
GDN_PROJ, ATTN_PROJ, MIXER_OUT = 8224, 5120, 2048

SIZES = {"0.8b": (1024, 3584), "2b": (2048, 6144)}


@dataclass
class Synth:
    index_json: str
    weights: np.ndarray  # uint8
    config: dict

    def save(self, directory) -> None:
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        self.weights.tofile(d / "weights.bin")
        (d / "index.json").write_text(self.index_json)


def _matrix_parts(kind: str, rows: int, k: int):
    el = rows * k
    if kind == "f16":
        return [("w", el * 2)]
    if kind == "q4":
        return [("w", el // 2), ("s", el // 16), ("z", el // 64)]
    if kind == "q4g64":
        return [("w", el // 2), ("s", el // 32), ("z", el // 32)]
    raise ValueError(kind)


def _fill_matrix(buf: np.ndarray, kind: str, part: str, rows: int, k: int, rng, std: float, scale_std: float):
    el = rows * k
    if kind == "f16":
        out = buf.view(np.float16)
        step = 1 << 24
        for i in range(0, el, step):
            n = min(step, el - i)
            out[i:i + n] = (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float16)
        return
    if part == "w":
        buf.view(np.uint32)[:] = rng.integers(0, 1 << 32, el // 8, dtype=np.uint64).astype(np.uint32)
        return
    if kind == "q4":
        if part == "s":
            sc = np.abs(rng.standard_normal(el // 32, dtype=np.float32) * np.float32(scale_std)).astype(np.float16)
            buf.view(np.float16)[:] = sc  # two f16 per u32, even block in the low half
        else:
            buf.view(np.uint32)[:] = 0x88888888
        return
    if part == "s":
        buf.view(np.float16)[:] = np.abs(rng.standard_normal(el // 64, dtype=np.float32) * np.float32(scale_std)).astype(np.float16)
    else:
        buf.view(np.float16)[:] = np.float16(8.0)


def build(hidden: int, intermediate: int, *, layers: int = 24, every: int = 4, vocab: int = VOCAB,
          kind: str = "f16", embed_kind: str = "f16", seed: int = 0, std: float = 0.02,
          scale_std: float = 0.01, theta: float = 1e7, tied: bool = True, threads: int = 8) -> Synth:
    """Builds the whole model in memory and returns (index.json text, weights bytes)."""
    plan = []  # (name, kind_or_None, part, rows, k, bytes, fill)
    matrices = {}

    def mat(name, rows, k, knd):
        matrices[name] = {"rows": rows, "k": k, "kind": knd}
        for part, nbytes in _matrix_parts(knd, rows, k):
            plan.append((f"{name}.{part}", knd, part, rows, k, nbytes))

    def vec(name, nbytes, fill):
        plan.append((name, None, fill, 0, 0, nbytes))

    mat("embed", vocab, hidden, embed_kind)
    for i in range(layers):
        attn = (i + 1) % every == 0
        p = f"layer{i}"
        vec(f"{p}.input_norm", hidden * 4, "ones")
        vec(f"{p}.post_norm", hidden * 4, "ones")
        mat(f"{p}.mixer_in", ATTN_PROJ if attn else GDN_PROJ, hidden, kind)
        mat(f"{p}.mixer_out", hidden, MIXER_OUT, kind)
        if attn:
            vec(f"{p}.attn_norms", 2048, "ones")
        else:
            vec(f"{p}.conv_w", 98304, "conv")
            vec(f"{p}.gdn_params", 640, "gdn")
        mat(f"{p}.gate_up", 2 * intermediate, hidden, kind)
        mat(f"{p}.down", hidden, intermediate, kind)
    vec("final_norm", hidden * 4, "ones")
    if tied:
        matrices["lm_head"] = dict(matrices["embed"])
    else:
        mat("lm_head", vocab, hidden, embed_kind)

    tensors = {}
    offset = 0
    for entry in plan:
        offset += (-offset) % ALIGN
        tensors[entry[0]] = {"offset": offset, "bytes": entry[5]}
        offset += entry[5]
    if tied:
        for part in ("w", "s", "z"):
            if f"embed.{part}" in tensors:
                tensors[f"lm_head.{part}"] = dict(tensors[f"embed.{part}"])
    weights = np.zeros(offset, np.uint8)

    def fill(idx):
        name, knd, part, rows, k, nbytes = plan[idx]
        rng = np.random.default_rng([seed, idx])
        off = tensors[name]["offset"]
        buf = weights[off:off + nbytes]
        if knd is not None:
            _fill_matrix(buf, knd, part, rows, k, rng, std, scale_std)
        elif part == "ones":
            buf.view(np.float32)[:] = 1.0
        elif part == "conv":
            buf.view(np.float32)[:] = rng.uniform(-0.5, 0.5, nbytes // 4).astype(np.float32)
        elif part == "gdn":
            v = buf.view(np.float32)
            v[:16] = 0.0
            v[16:32] = -0.5
            v[32:] = 1.0

    order = sorted(range(len(plan)), key=lambda i: -plan[i][5])
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(fill, order))

    config = {"layers": layers, "full_attention_every": every, "hidden": hidden, "intermediate": intermediate,
              "vocab": vocab, "rope_theta": theta, "rope_dim": 64}
    index = {"source": f"synthetic seed {seed}", "format_version": 1, "config": config,
             "matrices": matrices, "tensors": tensors}
    return Synth(json.dumps(index), weights, config)


def baseline_config(n: int) -> dict:
    """the benchmark configs 1-4 as build() keyword arguments plus the workload."""
    if n == 1:
        return dict(size="0.8b", kind="f16", seed=0, prompt=128, steps=128, batch=1)
    if n == 2:
        return dict(size="2b", kind="f16", seed=1, prompt=3968, steps=128, batch=1)
    if n == 3:
        return dict(size="2b", kind="q4g64", seed=2, prompt=1024, steps=256, batch=1)
    if n == 4:
        return dict(size="0.8b", kind="f16", seed=3, prompt=None, steps=64, batch=32)
    raise ValueError(n)


def build_config(n: int, **overrides) -> Synth:
    c = baseline_config(n)
    hidden, inter = SIZES[c["size"]]
    kw = dict(kind=c["kind"], seed=c["seed"])
    kw.update(overrides)
    return build(hidden, inter, **kw)


def prompt_ids(n: int, seed: int, vocab: int = VOCAB) -> np.ndarray:
    """n token ids uniform in [0, vocab) from `seed`."""
    return np.random.default_rng(seed).integers(0, vocab, n, dtype=np.uint32)
