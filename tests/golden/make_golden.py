"""Regenerates tests/golden/reference_checks.npz: expected outputs of the reference's own kernel
self-checks, restated independently of the oracle.

The reference (arlinamid/qwen-native-engine) ships no kernel golden vectors; its kernels are
pinned by CPU re-computations inside `run()` (kernels/src/lib.rs:865-896) on inputs from its
xorshift generator seeded 0x9E3779B97F4A7C15 (kernels/src/lib.rs:170-182, 872). This script
replays that input stream in pure Python, in the order `run()` draws it on an f16-capable GPU
(gemv f32 x3, gemv f16 / f16-split4 x6, gemm x3, gdn, attention, embed + argmax), and evaluates
the CPU reference formulas of check_gemv / check_gemm / check_gdn / check_attention /
check_embed_and_argmax (kernels/src/lib.rs:513-712) in float64 with numpy. The reference
itself cannot run here (Rust toolchain and a graphics adapter are absent), so these vectors are
the restated formulas, not recorded reference output.

Usage: python tests/golden/make_golden.py  (about a minute; writes the .npz next to this file)
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

MASK = (1 << 64) - 1
VOCAB = 248320
OUT = Path(__file__).resolve().parent / "reference_checks.npz"


class Rng:
    """xorshift64, kernels/src/lib.rs:170-182."""

    def __init__(self, seed: int):
        self.s = seed

    def next_u32(self) -> int:
        s = self.s
        s ^= (s << 13) & MASK
        s ^= s >> 7
        s ^= (s << 17) & MASK
        self.s = s
        return s >> 32

    def u32(self, n: int) -> np.ndarray:
        return np.array([self.next_u32() for _ in range(n)], dtype=np.uint32)

    def f32(self, n: int) -> np.ndarray:
        # (next_u32 >> 8) / 2^24 * 2 - 1, exact in f32 and f64
        return np.array([((self.next_u32() >> 8) / 16777216.0) * 2.0 - 1.0 for _ in range(n)], dtype=np.float64)


def f16(bits: np.ndarray) -> np.ndarray:
    return bits.astype(np.uint16).view(np.float16).astype(np.float64)


def dequant(w, s, z, rows, k) -> np.ndarray:
    """dequant_row for all rows (kernels/src/lib.rs:484-497), float64."""
    c = np.arange(k)
    W = w.reshape(rows, k // 8)
    q = (W[:, c // 8] >> (4 * (c % 8)).astype(np.uint32)) & 15
    blk = c // 32
    S = s.reshape(rows, k // 64)[:, blk // 2]
    scale = np.where(blk % 2 == 0, f16(S & 0xFFFF), f16(S >> 16))
    Z = z.reshape(rows, k // 256)[:, blk // 8]
    zp = (Z >> (4 * (blk % 8)).astype(np.uint32)) & 15
    return (q.astype(np.float64) - zp.astype(np.float64)) * scale


def silu(x):
    return x / (1.0 + np.exp(-x))


def qmat_inputs(rng: Rng, rows: int, k: int):
    w = rng.u32(rows * k // 8)
    s = (0x20002400 + (rng.u32(rows * k // 64) & 0x00FF00FF)).astype(np.uint32)
    z = rng.u32(rows * k // 256)
    return w, s, z


def check_gemv(rng: Rng, epi: str):
    out_rows, k = 37, 1024
    rows = out_rows * 2 if epi == "swiglu" else out_rows
    w, s, z = qmat_inputs(rng, rows, k)
    x = rng.f32(k)
    y0 = rng.f32(out_rows)
    d = dequant(w, s, z, rows, k) @ x
    if epi == "store":
        return d[:out_rows]
    if epi == "accumulate":
        return y0 + d[:out_rows]
    return silu(d[:out_rows]) * d[out_rows:]


def check_gemm(rng: Rng, epi: str):
    out_rows, k, count, batch = 70, 1024, 11, 16
    rows = out_rows * 2 if epi == "swiglu" else out_rows
    w, s, z = qmat_inputs(rng, rows, k)
    x = rng.f32(batch * k).reshape(batch, k)
    y0 = rng.f32(batch * out_rows).reshape(batch, out_rows)
    D = dequant(w, s, z, rows, k)
    res = []
    for t in range(count):
        d = D @ x[t]
        if epi == "store":
            res.append(d[:out_rows])
        elif epi == "accumulate":
            res.append(y0[t] + d[:out_rows])
        else:
            res.append(silu(d[:out_rows]) * d[out_rows:])
    return np.stack(res)


def check_gdn(rng: Rng):
    proj = rng.f32(8224)
    conv0 = rng.f32(6144 * 3)
    # derived inputs are computed in f32, as the reference does, then widened
    f = np.float32
    conv_w = (rng.f32(6144 * 4).astype(f) * f(0.5)).astype(np.float64)
    state0 = (rng.f32(16 * 16384).astype(f) * f(0.1)).astype(np.float64)
    prm = np.empty(160)
    for i in range(160):
        v = f(rng.f32(1)[0])
        prm[i] = v * f(4.0) if i < 16 else (f(-0.5) + v * f(0.4) if i < 32 else f(1.0) + v * f(0.3))
    c = np.arange(6144)
    conv = silu(conv0[c * 3] * conv_w[c * 4] + conv0[c * 3 + 1] * conv_w[c * 4 + 1] +
                conv0[c * 3 + 2] * conv_w[c * 4 + 2] + proj[c] * conv_w[c * 4 + 3])
    want_o = np.zeros(2048)
    want_state = state0.copy().reshape(16, 128, 128)
    S0 = state0.reshape(16, 128, 128)
    for h in range(16):
        q = conv[h * 128:(h + 1) * 128]
        k = conv[2048 + h * 128:2048 + (h + 1) * 128]
        v = conv[4096 + h * 128:4096 + (h + 1) * 128]
        qs = q / np.sqrt((q * q).sum() + 1e-6) * 0.08838834764
        ks = k / np.sqrt((k * k).sum() + 1e-6)
        g = np.exp(prm[16 + h] * np.log(1.0 + np.exp(proj[8192 + h] + prm[h])))
        beta = 1.0 / (1.0 + np.exp(-proj[8208 + h]))
        kq = (ks * qs).sum()
        sk = S0[h].T @ ks  # [t]
        sq = S0[h].T @ qs
        dv = beta * (v - g * sk)
        want_state[h] = g * S0[h] + np.outer(ks, dv)
        out = g * sq + dv * kq
        inv = 1.0 / np.sqrt((out * out).sum() / 128.0 + 1e-6)
        want_o[h * 128:(h + 1) * 128] = out * inv * silu(proj[6144 + h * 128:6144 + (h + 1) * 128]) * prm[32:160]
    return want_o, want_state.reshape(-1)


def check_attention(rng: Rng):
    pos = 5
    proj = rng.f32(5120)
    cache_len = 2 * 4096 * 256
    kc = rng.f32(cache_len).reshape(2, 4096, 256)
    vc = rng.f32(cache_len).reshape(2, 4096, 256)
    prm = (np.float32(1.0) + rng.f32(512).astype(np.float32) * np.float32(0.5)).astype(np.float64)

    def norm_rope(x, w):
        y = x / np.sqrt((x * x).sum() / 256.0 + 1e-6) * w
        i = np.arange(32)
        ang = pos * np.power(1e7, -(2.0 * i) / 64.0)
        a, b = y[:32].copy(), y[32:64].copy()
        y[:32] = a * np.cos(ang) - b * np.sin(ang)
        y[32:64] = b * np.cos(ang) + a * np.sin(ang)
        return y

    want = np.zeros(2048)
    for h in range(8):
        kvh = h // 4
        q = norm_rope(proj[h * 256:(h + 1) * 256], prm[:256])
        kcur = norm_rope(proj[4096 + kvh * 256:4096 + (kvh + 1) * 256], prm[256:])
        keys = kc[kvh, :pos + 1].copy()
        vals = vc[kvh, :pos + 1].copy()
        keys[pos] = kcur
        vals[pos] = proj[4608 + kvh * 256:4608 + (kvh + 1) * 256]
        sc = keys @ q * 0.0625
        e = np.exp(sc - sc.max())
        want[h * 256:(h + 1) * 256] = (e @ vals) / e.sum() / (1.0 + np.exp(-proj[2048 + h * 256:2048 + (h + 1) * 256]))
    return want


def check_embed_and_argmax(rng: Rng):
    rows, hidden = 300, 1024
    w, s, z = qmat_inputs(rng, rows, hidden)
    logits = rng.f32(VOCAB)
    logits[123457] = 9.0
    embed = dequant(w, s, z, rows, hidden)[7]
    tok = [int(np.argmax(logits)), 41 + 1]
    return embed, np.array(tok, dtype=np.uint32)


def main():
    rng = Rng(0x9E3779B97F4A7C15)
    probe = Rng(0x9E3779B97F4A7C15)
    out = {"rng_u32_head": probe.u32(16), "rng_f32_head": Rng(0x9E3779B97F4A7C15).f32(16).astype(np.float32)}
    names = []
    for f16_variant in (False, True):
        for epi in ("store", "accumulate", "swiglu"):
            for splits in ((1,) if not f16_variant else (1, 4)):
                name = f"gemv_{'f16' if f16_variant else 'f32'}_{epi}_split{splits}"
                out[name] = check_gemv(rng, epi).astype(np.float32)
                names.append(name)
    for epi in ("store", "accumulate", "swiglu"):
        out[f"gemm_{epi}"] = check_gemm(rng, epi).astype(np.float32)
    o, st = check_gdn(rng)
    out["gdn_output"] = o.astype(np.float32)
    out["gdn_state_sample"] = st[::61].astype(np.float32)
    out["gdn_state_head_sums"] = st.reshape(16, -1).sum(axis=1)
    out["attention"] = check_attention(rng).astype(np.float32)
    e, tok = check_embed_and_argmax(rng)
    out["embed"] = e.astype(np.float32)
    out["argmax_tok"] = tok
    out["rng_state_end"] = np.array([rng.s], dtype=np.uint64)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes), {len(names)} gemv checks")


if __name__ == "__main__":
    main()
