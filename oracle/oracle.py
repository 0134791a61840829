"""ctypes binding of the CPU oracle (liboracle.so built from qne_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
cpu-baseline leg as the checker. The engine never imports it.
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "liboracle.so"
KINDS = {"f16": 0, "q4": 1, "q4g64": 2}
MAX_CTX = 4096


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built (make -C oracle)")
    lib = C.CDLL(str(LIB_PATH))
    P, I, F = C.c_void_p, C.c_int, C.c_float
    sig = {
        "oracle_f16_to_f32_ref": (F, [C.c_uint16]),
        "oracle_dequant_rows": (None, [I, P, P, P, I, I, I, I, P]),
        "oracle_gemv": (None, [I, P, P, P, I, I, P, P, I]),
        "oracle_rmsnorm": (None, [P, P, I, P]),
        "oracle_gdn_step": (None, [P, P, P, P, P, P]),
        "oracle_rope_table": (None, [C.c_double, P]),
        "oracle_attention_step": (None, [P, P, P, I, P, P, I, P]),
        "oracle_argmax": (C.c_uint32, [P, C.c_long]),
        "oracle_round_f16": (F, [F]),
        "oracle_threads": (I, []),
        "oracle_model_new": (P, [I, I, I, I, I, C.c_double, I, C.POINTER(P), C.POINTER(I)]),
        "oracle_model_free": (None, [P]),
        "oracle_model_reset": (None, [P]),
        "oracle_model_step": (None, [P, C.c_uint32, I, P]),
        "oracle_model_state": (I, [P, I, P, P, I]),
        "oracle_rng_u32": (None, [C.POINTER(C.c_uint64), C.c_long, P]),
        "oracle_rng_f32": (None, [C.POINTER(C.c_uint64), C.c_long, P]),
        "oracle_model_prefill": (I, [P, P, I, I, P]),
        "oracle_model_snapshot": (None, [P, C.POINTER(P)]),
        "oracle_model_restore": (I, [P, P]),
        "oracle_snapshot_free": (None, [P]),
        "oracle_model_fill_synthetic": (None, [P, I, C.c_uint64]),
        "oracle_gemm_tokens": (None, [I, P, P, P, I, I, P, I, P, I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _p(a):
    return None if a is None else a.ctypes.data


class Rng:
    """The reference's xorshift64 (kernels/src/lib.rs:170-182), generated in C."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(seed)

    def u32(self, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        lib.oracle_rng_u32(C.byref(self.state), n, _p(out))
        return out

    def f32(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib.oracle_rng_f32(C.byref(self.state), n, _p(out))
        return out


def threads() -> int:
    return int(lib.oracle_threads())


def f16_to_f32_ref(h: int) -> float:
    return float(lib.oracle_f16_to_f32_ref(h))


def dequant_rows(kind: str, w, s, z, rows: int, k: int, row0: int, nrows: int) -> np.ndarray:
    out = np.empty((nrows, k), np.float32)
    lib.oracle_dequant_rows(KINDS[kind], _p(w), _p(s), _p(z), rows, k, row0, nrows, _p(out))
    return out


def gemv(kind: str, w, s, z, rows: int, k: int, x: np.ndarray, y: np.ndarray, epilogue: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    lib.oracle_gemv(KINDS[kind], _p(w), _p(s), _p(z), rows, k, _p(x), _p(y), epilogue)
    return y


def rmsnorm(x: np.ndarray, g: np.ndarray) -> np.ndarray:
    y = np.empty_like(x)
    lib.oracle_rmsnorm(_p(x), _p(g), x.size, _p(y))
    return y


def gdn_step(proj, conv_state, conv_w, state, params) -> np.ndarray:
    """Reference layouts: conv_state [6144*3] (oldest first), state [16][128][128]. Updates both."""
    out = np.empty(2048, np.float32)
    lib.oracle_gdn_step(_p(proj), _p(conv_state), _p(conv_w), _p(state), _p(params), _p(out))
    return out


def rope_table(theta: float = 1e7) -> np.ndarray:
    t = np.empty(2 * MAX_CTX * 32, np.float32)
    lib.oracle_rope_table(theta, _p(t))
    return t


def attention_step(proj, kc, vc, pos: int, norms, rope, kv_f16: bool) -> np.ndarray:
    """kc, vc: [2][4096][256] f32 contiguous caches; the current K/V are written at `pos`."""
    out = np.empty(2048, np.float32)
    lib.oracle_attention_step(_p(proj), _p(kc), _p(vc), pos, _p(norms), _p(rope), 1 if kv_f16 else 0, _p(out))
    return out


def gemm_tokens(kind: str, w, s, z, rows: int, k: int, x: np.ndarray, y: np.ndarray, epilogue: int) -> np.ndarray:
    """The batched prefill's matrix product: y[n][out] (=, +=, SwiGLU) for token rows x[n][k]."""
    x = np.ascontiguousarray(x, np.float32)
    lib.oracle_gemm_tokens(KINDS[kind], _p(w), _p(s), _p(z), rows, k, _p(x), x.shape[0], _p(y), epilogue)
    return y


def argmax(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return int(lib.oracle_argmax(_p(x), x.size))


class OracleModel:
    """The whole decode step on the CPU over the same weights.bin + index.json."""

    def __init__(self, index_json: str, weights: np.ndarray, kv_f16: bool = True):
        idx = json.loads(index_json)
        c = idx["config"]
        self.vocab = c["vocab"]
        self.layers = c["layers"]
        self.weights = np.ascontiguousarray(weights).view(np.uint8)
        base = self.weights.ctypes.data
        t = idx["tensors"]
        m = idx["matrices"]
        ptrs, kinds = [], []

        def tensor(name):
            return base + t[name]["offset"] if name in t else None

        def mat(name):
            kinds.append(KINDS[m[name].get("kind", "q4")])
            ptrs.extend([tensor(f"{name}.w"), tensor(f"{name}.s"), tensor(f"{name}.z")])

        mat("embed")
        mat("lm_head")
        ptrs.append(tensor("final_norm"))
        for i in range(c["layers"]):
            p = f"layer{i}"
            attn = (i + 1) % c["full_attention_every"] == 0
            ptrs.extend([tensor(f"{p}.input_norm"), tensor(f"{p}.post_norm")])
            for part in ("mixer_in", "mixer_out", "gate_up", "down"):
                mat(f"{p}.{part}")
            if attn:
                ptrs.extend([tensor(f"{p}.attn_norms"), None])
            else:
                ptrs.extend([tensor(f"{p}.conv_w"), tensor(f"{p}.gdn_params")])
        # per-layer matrix order in the C side: in, out, gate_up, down, then norms
        self._ptrs = (C.c_void_p * len(ptrs))(*ptrs)
        self._kinds = (C.c_int * len(kinds))(*kinds)
        inter = c.get("intermediate") or (3584 if c["hidden"] == 1024 else 6144)
        self._h = lib.oracle_model_new(c["layers"], c["full_attention_every"], c["hidden"], inter, c["vocab"],
                                       float(c["rope_theta"]), 1 if kv_f16 else 0, self._ptrs, self._kinds)
        self.every = c["full_attention_every"]
        self._saved = None

    def close(self):
        if getattr(self, "_saved", None):
            lib.oracle_snapshot_free(self._saved)
            self._saved = None
        if self._h:
            lib.oracle_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        lib.oracle_model_reset(self._h)

    def step(self, token: int, pos: int, want_logits: bool = True):
        out = np.empty(self.vocab, np.float32) if want_logits else None
        lib.oracle_model_step(self._h, int(token), int(pos), _p(out))
        return out

    def prefill(self, ids, start: int = 0):
        """Runs ids from `start`; returns the logits after the last one."""
        ids = list(ids)
        for i, t in enumerate(ids[:-1]):
            self.step(t, start + i, want_logits=False)
        return self.step(ids[-1], start + len(ids) - 1)

    def prefill_batched(self, ids, start: int = 0, want_logits: bool = True):
        """The same tokens as prefill() through the batched CPU path (all tokens of each matrix
        product at once, GDN and attention over the whole run): seconds for a 4000-token prompt
        instead of minutes. Returns the logits after the last id (or None)."""
        a = np.ascontiguousarray(np.asarray(list(ids), dtype=np.uint32))
        out = np.empty(self.vocab, np.float32) if want_logits else None
        if lib.oracle_model_prefill(self._h, _p(a), a.size, int(start), _p(out)) != 0:
            raise ValueError(f"prefill of {a.size} tokens from {start} exceeds the {MAX_CTX}-token context")
        return out

    def snapshot(self):
        saved = C.c_void_p(getattr(self, "_saved", None) or 0)
        lib.oracle_model_snapshot(self._h, C.byref(saved))
        self._saved = saved.value

    def restore(self):
        if lib.oracle_model_restore(self._h, getattr(self, "_saved", None)) != 0:
            raise ValueError("no snapshot taken")

    def fill_synthetic(self, length: int, seed: int):
        """Seeded synthetic KV history for positions [0, length) and GDN states (throughput samples)."""
        lib.oracle_model_fill_synthetic(self._h, int(length), int(seed))

    def greedy(self, first_logits: np.ndarray, start_pos: int, n: int):
        """Greedy continuation: returns (ids, per-step logits margins) for n tokens."""
        ids, margins = [], []
        logits = first_logits
        pos = start_pos
        for _ in range(n):
            tok = argmax(logits)
            top2 = np.partition(logits, -2)[-2:]
            margins.append(float(abs(top2[1] - top2[0])))
            ids.append(tok)
            logits = self.step(tok, pos)
            pos += 1
        return ids, margins

    def state(self, layer: int, length: int = 0):
        attn = (layer + 1) % self.every == 0
        if attn:
            a = np.empty((2, length, 256), np.float32)
            b = np.empty((2, length, 256), np.float32)
        else:
            a = np.empty(6144 * 3, np.float32)
            b = np.empty(16 * 16384, np.float32)
        lib.oracle_model_state(self._h, layer, _p(a), _p(b), length)
        return a, b
