"""Inputs of the reference's kernel self-checks (kernels/src/lib.rs:513-712), replayed from its
xorshift stream in the order run() (kernels/src/lib.rs:874-889) draws them, and the tolerances
those checks use. Shared by the oracle pin tests and the GPU parity tests."""
from dataclasses import dataclass

import numpy as np

from oracle import oracle

SEED = 0x9E3779B97F4A7C15
VOCAB = 248320
GEMV_ORDER = [("f32", "store", 1), ("f32", "accumulate", 1), ("f32", "swiglu", 1),
              ("f16", "store", 1), ("f16", "store", 4), ("f16", "accumulate", 1), ("f16", "accumulate", 4),
              ("f16", "swiglu", 1), ("f16", "swiglu", 4)]
EPI = {"store": 0, "accumulate": 1, "swiglu": 2}
# Reference tolerances: gemv f32 1e-4 (lib.rs:538), gdn output 1e-3 / state 1e-4 (lib.rs:625-626),
# attention 1e-3 (lib.rs:676), embed 1e-6 (lib.rs:709).
TOL_GEMV, TOL_GDN_OUT, TOL_GDN_STATE, TOL_ATTN, TOL_EMBED = 1e-4, 1e-3, 1e-4, 1e-3, 1e-6


def rel_err(got, want) -> float:
    """kernels/src/lib.rs:499-507: max |got - want| / max(1e-6, max |want|); non-finite -> inf."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    if got.shape != want.shape or not np.all(np.isfinite(got)) or not np.all(np.isfinite(want)):
        return float("inf")
    return float(np.abs(got - want).max() / max(1e-6, np.abs(want).max()))


@dataclass
class GemvCase:
    name: str
    epilogue: str
    rows: int
    k: int
    w: np.ndarray
    s: np.ndarray
    z: np.ndarray
    x: np.ndarray
    y0: np.ndarray


def _qmat(rng, rows, k):
    w = rng.u32(rows * k // 8)
    s = (0x20002400 + (rng.u32(rows * k // 64) & 0x00FF00FF)).astype(np.uint32)
    z = rng.u32(rows * k // 256)
    return w, s, z


def replay():
    """Returns a dict with every check's inputs, in draw order."""
    rng = oracle.Rng(SEED)
    cases = {"gemv": [], "gemm": []}
    for variant, epi, splits in GEMV_ORDER:
        out_rows, k = 37, 1024
        rows = out_rows * 2 if epi == "swiglu" else out_rows
        w, s, z = _qmat(rng, rows, k)
        x = rng.f32(k)
        y0 = rng.f32(out_rows)
        cases["gemv"].append(GemvCase(f"gemv_{variant}_{epi}_split{splits}", epi, rows, k, w, s, z, x, y0))
    for epi in ("store", "accumulate", "swiglu"):
        out_rows, k = 70, 1024
        rows = out_rows * 2 if epi == "swiglu" else out_rows
        w, s, z = _qmat(rng, rows, k)
        x = rng.f32(16 * k).reshape(16, k)
        y0 = rng.f32(16 * out_rows).reshape(16, out_rows)
        cases["gemm"].append(GemvCase(f"gemm_{epi}", epi, rows, k, w, s, z, x, y0))
    g = {}
    g["proj"] = rng.f32(8224)
    g["conv0"] = rng.f32(6144 * 3)
    g["conv_w"] = rng.f32(6144 * 4) * np.float32(0.5)
    g["state0"] = rng.f32(16 * 16384) * np.float32(0.1)
    prm = np.empty(160, np.float32)
    for i in range(160):
        v = rng.f32(1)[0]
        prm[i] = v * np.float32(4.0) if i < 16 else (np.float32(-0.5) + v * np.float32(0.4) if i < 32 else np.float32(1.0) + v * np.float32(0.3))
    g["params"] = prm
    cases["gdn"] = g
    a = {"pos": 5, "proj": rng.f32(5120)}
    a["kc"] = rng.f32(2 * 4096 * 256)
    a["vc"] = rng.f32(2 * 4096 * 256)
    a["norms"] = np.float32(1.0) + rng.f32(512) * np.float32(0.5)
    cases["attention"] = a
    e = {}
    e["w"], e["s"], e["z"] = _qmat(rng, 300, 1024)
    logits = rng.f32(VOCAB)
    logits[123457] = 9.0
    e["logits"] = logits
    cases["embed"] = e
    cases["rng_state_end"] = int(rng.state.value)
    return cases
