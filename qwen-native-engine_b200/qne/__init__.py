"""Python mirror of the `qwen-kernels` decoder API over the libqne C ABI (include/qne.h).

`Model` follows `kernels/src/model.rs` (struct Model): load / reset / prefill /
prefill_batched / prefill_from / prefill_chunk / logits / step / snapshot / restore /
last_token / decode / dispatches_per_token / profile-free adapter string, with the same
argument meanings and the same failures (context limit, bad index.json, no snapshot), raised
as `QneError`. `ModelTiles.validate` mirrors kernels/src/model.rs:101-109.

Operators (`gemv`, `rmsnorm_gemv`, `dequant_rows`, `argmax`, `gdn_step`, `attention_step`,
`kv_gather`, `embed`) take device tensors (torch is used only for device memory and streams)
and call the sm_100a kernels directly.

The shared library is opened on first use (importing the package loads no native code); the
first call raises ImportError if libqne.so is missing, and no operation falls back to another
implementation.
"""
from __future__ import annotations

import ctypes as C
import weakref
import os
from pathlib import Path

import numpy as np

MAX_CONTEXT = 4096
PAGE_TOKENS = 16
PAGES_PER_SEQ = MAX_CONTEXT // PAGE_TOKENS
PREFILL_CHUNK_TOKENS = 64  # tokens per batched prefill chunk
KIND_F16, KIND_Q4, KIND_Q4G64 = 0, 1, 2
KINDS = {"f16": KIND_F16, "q4": KIND_Q4, "q4g64": KIND_Q4G64}
EPI_STORE, EPI_ACCUMULATE, EPI_SWIGLU = 0, 1, 2
EPILOGUES = {"store": EPI_STORE, "accumulate": EPI_ACCUMULATE, "swiglu": EPI_SWIGLU}

_ERRORS = {-1: "EINVAL", -2: "ERANGE_CTX", -3: "EFORMAT", -4: "ECUDA", -5: "ETIMEOUT",
           -6: "ENOSNAP", -7: "ENOMEM"}

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libqne.so"


class QneError(RuntimeError):
    """A failed libqne call: `code` is the negative QNE_E* status, `name` its symbol."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.name = _ERRORS.get(code, str(code))
        super().__init__(f"{self.name}: {message}")


class _Matrix(C.Structure):
    _fields_ = [("kind", C.c_int32), ("rows", C.c_int32), ("k", C.c_int32), ("pad", C.c_int32),
                ("w", C.c_void_p), ("s", C.c_void_p), ("z", C.c_void_p)]


class _Sampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float), ("seed", C.c_uint64),
                ("presence_penalty", C.c_float)]


class _ProfileEntry(C.Structure):
    _fields_ = [("label", C.c_char * 48), ("ms", C.c_double), ("dispatches", C.c_uint32), ("pad", C.c_uint32)]


class _Info(C.Structure):
    _fields_ = [("layers", C.c_int32), ("hidden", C.c_int32), ("intermediate", C.c_int32),
                ("vocab", C.c_int32), ("weight_kind", C.c_int32), ("embed_kind", C.c_int32),
                ("tied_lm_head", C.c_int32), ("device", C.c_int32), ("weight_bytes", C.c_uint64),
                ("device_bytes", C.c_uint64)]


def _load_lib() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"libqne.so is not built ({LIB_PATH}); run __graft_entry__.build()")
    lib = C.CDLL(str(LIB_PATH))
    P, U32, I32, SZ = C.c_void_p, C.c_uint32, C.c_int, C.c_size_t
    U32P = C.POINTER(C.c_uint32)
    FP = C.POINTER(C.c_float)
    sigs = {
        "qne_last_error": (C.c_char_p, []),
        "qne_version": (C.c_char_p, []),
        "qne_kernel_launches": (C.c_uint64, []),
        "qne_model_load": (I32, [C.c_char_p, SZ, P, SZ, I32, C.POINTER(P)]),
        "qne_model_load_ex": (I32, [C.c_char_p, SZ, P, SZ, I32, U32, C.POINTER(P)]),
        "qne_model_free": (None, [P]),
        "qne_model_info_get": (I32, [P, C.POINTER(_Info)]),
        "qne_model_set_stream": (I32, [P, P]),
        "qne_model_set_fused": (I32, [P, I32]),
        "qne_model_fused": (I32, [P]),
        "qne_model_set_path": (I32, [P, I32]),
        "qne_model_path": (I32, [P]),
        "qne_model_set_phase_trace": (I32, [P, I32]),
        "qne_model_test_barrier_timeout": (I32, [P, U32]),
        "qne_profile_token": (I32, [P, C.POINTER(_ProfileEntry), SZ, C.POINTER(SZ)]),
        "qne_model_phase_trace": (I32, [P, P, SZ, C.POINTER(SZ), C.POINTER(SZ)]),
        "qne_adapter": (C.c_char_p, [P]),
        "qne_dispatches_per_token": (SZ, [P]),
        "qne_prefill_chunk_batched": (I32, [P]),
        "qne_validate_tiles": (I32, [C.c_char_p, SZ]),
        "qne_reset": (I32, [P]),
        "qne_prefill": (I32, [P, U32P, U32]),
        "qne_prefill_chunk": (I32, [P, U32P, U32, U32, I32]),
        "qne_logits": (I32, [P, FP, SZ]),
        "qne_step": (I32, [P, U32, U32, FP, SZ]),
        "qne_snapshot": (I32, [P]),
        "qne_restore": (I32, [P]),
        "qne_last_token": (I32, [P, U32P, U32P]),
        "qne_decode": (I32, [P, U32, U32, U32P, U32, U32P, U32P]),
        "qne_decode_async": (I32, [P, U32]),
        "qne_step_async": (I32, [P, U32, U32]),
        "qne_sync": (I32, [P, U32]),
        "qne_logits_device": (P, [P]),
        "qne_model_matrix": (I32, [P, C.c_char_p, C.POINTER(_Matrix)]),
        "qne_model_tensor": (I32, [P, C.c_char_p, C.POINTER(P)]),
        "qne_batch_create": (I32, [P, U32, U32, C.POINTER(P)]),
        "qne_batch_free": (None, [P]),
        "qne_batch_set_page_table": (I32, [P, U32P, SZ]),
        "qne_batch_reset": (I32, [P]),
        "qne_batch_step": (I32, [P, U32P, U32P, FP, U32P]),
        "qne_batch_decode_async": (I32, [P, U32]),
        "qne_batch_tokens": (I32, [P, U32P, U32P]),
        "qne_batch_fill_synthetic": (I32, [P, U32, U32, U32, C.c_uint64]),
        "qne_batch_sync": (I32, [P, U32]),
        "qne_gemv": (I32, [C.POINTER(_Matrix), P, P, I32, P]),
        "qne_rmsnorm_gemv": (I32, [C.POINTER(_Matrix), P, P, C.c_float, P, I32, P]),
        "qne_gemv_ex": (I32, [C.POINTER(_Matrix), P, P, I32, I32, I32, P]),
        "qne_gemm_scratch_bytes": (SZ, [C.POINTER(_Matrix), I32]),
        "qne_gemm": (I32, [C.POINTER(_Matrix), P, I32, P, I32, P, SZ, P]),
        "qne_gemm_ex": (I32, [C.POINTER(_Matrix), P, I32, P, I32, I32, P]),
        "qne_gemm_noalloc": (I32, [C.POINTER(_Matrix), P, I32, P, I32, P]),
        "qne_dequant_rows": (I32, [C.POINTER(_Matrix), I32, I32, P, P]),
        "qne_embed": (I32, [C.POINTER(_Matrix), P, P, P]),
        "qne_argmax_scratch_bytes": (SZ, [U32]),
        "qne_argmax": (I32, [P, U32, P, P, SZ, P]),
        "qne_gdn_step": (I32, [P, P, P, P, P, P, P, I32, P]),
        "qne_attention_scratch_bytes": (SZ, [I32]),
        "qne_attention_step": (I32, [P, P, C.c_double, P, U32, P, P, P, I32, P, SZ, P]),
        "qne_attention_step_ex": (I32, [P, P, C.c_double, P, U32, P, P, P, I32, P, SZ, I32, P]),
        "qne_kv_gather": (I32, [P, P, U32, P, P, P]),
        "qne_bandwidth_probe": (I32, [P, SZ, P, P]),
        "qne_dispatch_cost": (I32, [U32, I32, P, P, C.POINTER(C.c_double)]),
        "qne_sampler_create": (I32, [P, C.POINTER(_Sampling), C.POINTER(P)]),
        "qne_sampler_free": (None, [P]),
        "qne_sampler_sample": (I32, [P, U32P, U32, C.c_int32, C.c_float, U32P]),
        "qne_sampler_sample_device": (I32, [P, P, U32P, U32, C.c_int32, C.c_float, U32P]),
        "qne_step_sample": (I32, [P, P, U32, U32, U32P, U32, C.c_int32, C.c_float, U32P]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class _LazyLib:
    """libqne.so, opened on first use: importing `qne` (for `qne.synth`, say) maps no native code,
    and the first call of any entry point raises ImportError if the library is not built."""

    _cdll: C.CDLL | None = None

    def __getattr__(self, name: str):
        if _LazyLib._cdll is None:
            _LazyLib._cdll = _load_lib()
        return getattr(_LazyLib._cdll, name)


lib = _LazyLib()


def _check(status: int) -> None:
    if status != 0:
        raise QneError(status, lib.qne_last_error().decode(errors="replace"))


def kernel_launches() -> int:
    """Kernels libqne has launched in this process."""
    return int(lib.qne_kernel_launches())


def version() -> str:
    return lib.qne_version().decode()


def _u32_array(values) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(values, dtype=np.uint32))


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


class ModelTiles:
    """The reference's per-matrix tile profile (kernels/src/model.rs:89-145). The CUDA kernels
    pick their own shapes; profiles are accepted and validated for API compatibility."""

    @staticmethod
    def validate(profile_json: str) -> None:
        b = profile_json.encode()
        _check(lib.qne_validate_tiles(b, len(b)))


LOAD_ANY_SHAPE = 1


class Model:
    """A loaded decoder on one GPU (kernels/src/model.rs:147-450).

    Like the reference's Model::load, only the Qwen3.5-0.8B and -2B architectures load; any other
    raises QneError(EFORMAT, "unsupported model architecture: ..."). `any_shape=True`
    (qne_model_load_ex with QNE_LOAD_ANY_SHAPE) also accepts smaller layer counts, vocabularies
    and widths, as the tests' small models need."""

    def __init__(self, index_json, weights, device: int = 0, any_shape: bool = False):
        if isinstance(index_json, str):
            index_json = index_json.encode()
        w = weights
        if isinstance(w, (bytes, bytearray)):
            buf = (C.c_char * len(w)).from_buffer_copy(w) if isinstance(w, bytes) else (C.c_char * len(w)).from_buffer(w)
            ptr, n = C.addressof(buf), len(w)
        else:
            arr = np.ascontiguousarray(w).view(np.uint8).reshape(-1)
            ptr, n = arr.ctypes.data, arr.nbytes
        h = C.c_void_p()
        if any_shape:
            _check(lib.qne_model_load_ex(index_json, len(index_json), C.c_void_p(ptr), n, device, LOAD_ANY_SHAPE,
                                         C.byref(h)))
        else:
            _check(lib.qne_model_load(index_json, len(index_json), C.c_void_p(ptr), n, device, C.byref(h)))
        self._h = h
        info = _Info()
        _check(lib.qne_model_info_get(self._h, C.byref(info)))
        self.layers = info.layers
        self.hidden = info.hidden
        self.intermediate = info.intermediate
        self.vocab = info.vocab
        self.weight_kind = info.weight_kind
        self.embed_kind = info.embed_kind
        self.tied_lm_head = bool(info.tied_lm_head)
        self.device = info.device
        self.weight_bytes = int(info.weight_bytes)
        self.device_bytes = int(info.device_bytes)
        self.adapter = lib.qne_adapter(self._h).decode()

    @classmethod
    def load(cls, index_json, weights, device: int = 0, any_shape: bool = False) -> "Model":
        return cls(index_json, weights, device, any_shape)

    def close(self) -> None:
        for ref in getattr(self, "_samplers", []):  # samplers are freed before their model
            smp = ref()
            if smp is not None:
                smp.close()
        if getattr(self, "_h", None):
            lib.qne_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- kernels/src/model.rs API ------------------------------------------------------------
    def dispatches_per_token(self) -> int:
        return int(lib.qne_dispatches_per_token(self._h))

    def reset(self) -> None:
        _check(lib.qne_reset(self._h))

    def prefill(self, ids) -> None:
        a = _u32_array(ids)
        _check(lib.qne_prefill(self._h, _u32p(a), len(a)))

    def prefill_batched(self, ids) -> None:
        self.prefill_from(ids, 0)

    def prefill_from(self, ids, start: int) -> None:
        self.prefill_chunk(ids, start, True)

    @property
    def prefill_batched_supported(self) -> bool:
        """Whether prefill_chunk runs 64-token batched chunks on this model (f16 or int4 weights)."""
        return bool(lib.qne_prefill_chunk_batched(self._h))

    def prefill_chunk(self, ids, start: int, finish_logits: bool) -> None:
        a = _u32_array(ids)
        _check(lib.qne_prefill_chunk(self._h, _u32p(a), len(a), start, 1 if finish_logits else 0))

    def logits(self, out: np.ndarray | None = None) -> np.ndarray:
        out = np.empty(self.vocab, np.float32) if out is None else out
        _check(lib.qne_logits(self._h, _fp(out), out.size))
        return out

    def step(self, token: int, pos: int, out: np.ndarray | None = None) -> np.ndarray:
        out = np.empty(self.vocab, np.float32) if out is None else out
        _check(lib.qne_step(self._h, token, pos, _fp(out), out.size))
        return out

    def step_sample(self, sampler: "Sampler", token: int, pos: int, mask=None, bias_token: int = -1,
                    bias: float = 0.0) -> int:
        """qne_step_sample: one step, then a draw on the device; returns only the token."""
        words, n = _mask_words(mask)
        out = C.c_uint32()
        _check(lib.qne_step_sample(self._h, sampler._h, token, pos, _u32p(words) if words is not None else None, n,
                                   bias_token, float(bias), C.byref(out)))
        return int(out.value)

    def profile_token(self) -> dict[str, float]:
        """Model::profile_token: consumes one greedy token; milliseconds per dispatch label, each
        kernel timed alone (no overlap with its neighbours)."""
        n = C.c_size_t()
        cap = 64
        buf = (_ProfileEntry * cap)()
        _check(lib.qne_profile_token(self._h, buf, cap, C.byref(n)))
        return {buf[i].label.decode(): buf[i].ms for i in range(min(n.value, cap))}

    def snapshot(self) -> None:
        _check(lib.qne_snapshot(self._h))

    def restore(self) -> None:
        _check(lib.qne_restore(self._h))

    def last_token(self) -> tuple[int, int]:
        t, p = C.c_uint32(), C.c_uint32()
        _check(lib.qne_last_token(self._h, C.byref(t), C.byref(p)))
        return int(t.value), int(p.value)

    def decode(self, n: int, window: int = 1, stop=()) -> list[int]:
        s = _u32_array(list(stop) or [0])
        out = np.zeros(max(n, 1), np.uint32)
        cnt = C.c_uint32()
        _check(lib.qne_decode(self._h, n, window, _u32p(s), len(stop), _u32p(out), C.byref(cnt)))
        return [int(x) for x in out[: cnt.value]]

    # -- engine extensions -------------------------------------------------------------------
    def decode_async(self, steps: int) -> None:
        _check(lib.qne_decode_async(self._h, steps))

    def step_async(self, token: int, pos: int) -> None:
        _check(lib.qne_step_async(self._h, token, pos))

    def sync(self, timeout_ms: int = 600_000) -> None:
        _check(lib.qne_sync(self._h, timeout_ms))

    def set_stream(self, stream_handle: int | None) -> None:
        _check(lib.qne_model_set_stream(self._h, C.c_void_p(stream_handle or 0)))

    def set_fused(self, enable: bool) -> None:
        """One fused cooperative launch per layer (True) or one kernel per operation (False)."""
        _check(lib.qne_model_set_fused(self._h, 1 if enable else 0))

    @property
    def fused(self) -> bool:
        return bool(lib.qne_model_fused(self._h))

    PATHS = {"operations": 0, "layers": 1, "token": 2}

    def set_path(self, path: str) -> None:
        """Launch path of a token: "operations" (one kernel per operation), "layers" (one fused
        launch per layer) or "token" (one launch per token)."""
        _check(lib.qne_model_set_path(self._h, self.PATHS[path]))

    @property
    def path(self) -> str:
        n = int(lib.qne_model_path(self._h))
        return {v: k for k, v in self.PATHS.items()}[n]

    def set_phase_trace(self, enable: bool) -> None:
        _check(lib.qne_model_set_phase_trace(self._h, 1 if enable else 0))

    def test_barrier_timeout(self, limit_us: int) -> None:
        """Fused path test hook: every grid-barrier wait runs out after limit_us (0 = off)."""
        _check(lib.qne_model_test_barrier_timeout(self._h, int(limit_us)))

    def phase_trace(self) -> np.ndarray:
        """Last token's fused-path timestamps, shape [layers, ctas, 32] (ns, %globaltimer)."""
        n, ctas = C.c_size_t(), C.c_size_t()
        _check(lib.qne_model_phase_trace(self._h, None, 0, C.byref(n), C.byref(ctas)))
        out = np.zeros(self.layers * ctas.value * 32, np.uint64)
        _check(lib.qne_model_phase_trace(self._h, out.ctypes.data, out.size, C.byref(n), C.byref(ctas)))
        return out.reshape(self.layers, ctas.value, 32)

    def matrix(self, name: str) -> _Matrix:
        """Device descriptor of a loaded matrix (index.json name)."""
        m = _Matrix()
        _check(lib.qne_model_matrix(self._h, name.encode(), C.byref(m)))
        return m

    def tensor_ptr(self, name: str) -> int:
        p = C.c_void_p()
        _check(lib.qne_model_tensor(self._h, name.encode(), C.byref(p)))
        return int(p.value)

    def logits_device_ptr(self) -> int:
        return int(lib.qne_logits_device(self._h) or 0)


class Batch:
    """Independent sequences decoded together on one model's weights."""

    def __init__(self, model: Model, batch: int, pool_pages: int | None = None):
        self.model = model
        self.batch = batch
        self.pool_pages = pool_pages if pool_pages is not None else batch * PAGES_PER_SEQ
        h = C.c_void_p()
        _check(lib.qne_batch_create(model._h, batch, self.pool_pages, C.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.qne_batch_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_page_table(self, table) -> None:
        a = _u32_array(table).reshape(-1)
        _check(lib.qne_batch_set_page_table(self._h, _u32p(a), a.size))

    def reset(self) -> None:
        _check(lib.qne_batch_reset(self._h))

    def step(self, tokens, pos, want_logits: bool = False):
        t, p = _u32_array(tokens), _u32_array(pos)
        nxt = np.zeros(self.batch, np.uint32)
        lg = np.empty((self.batch, self.model.vocab), np.float32) if want_logits else None
        _check(lib.qne_batch_step(self._h, _u32p(t), _u32p(p), _fp(lg) if lg is not None else None, _u32p(nxt)))
        return (nxt, lg) if want_logits else nxt

    def decode_async(self, steps: int) -> None:
        _check(lib.qne_batch_decode_async(self._h, steps))

    def tokens(self):
        t = np.zeros(self.batch, np.uint32)
        p = np.zeros(self.batch, np.uint32)
        _check(lib.qne_batch_tokens(self._h, _u32p(t), _u32p(p)))
        return t, p

    def fill_synthetic(self, seq: int, length: int, token: int, seed: int) -> None:
        _check(lib.qne_batch_fill_synthetic(self._h, seq, length, token, seed))

    def sync(self, timeout_ms: int = 600_000) -> None:
        _check(lib.qne_batch_sync(self._h, timeout_ms))


# ---------------------------------------------------------------------------------------------
# Operators on device tensors (torch tensors or raw pointers)
# ---------------------------------------------------------------------------------------------
def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return int(t.data_ptr())


def _stream(stream) -> C.c_void_p:
    if stream is None:
        try:
            import torch
            return C.c_void_p(torch.cuda.current_stream().cuda_stream)
        except Exception:
            return C.c_void_p(0)
    return C.c_void_p(int(stream))


def matrix(kind, rows: int, k: int, w, s=None, z=None) -> _Matrix:
    kind = KINDS[kind] if isinstance(kind, str) else int(kind)
    return _Matrix(kind, rows, k, 0, _ptr(w), _ptr(s), _ptr(z))


def gemv(m: _Matrix, x, y, epilogue="store", stream=None) -> None:
    epi = EPILOGUES[epilogue] if isinstance(epilogue, str) else int(epilogue)
    _check(lib.qne_gemv(C.byref(m), _ptr(x), _ptr(y), epi, _stream(stream)))


def gemv_ex(m: _Matrix, x, y, epilogue="store", variant: int = 0, ctas_per_sm: int = 2, stream=None) -> None:
    """gemv with an explicit kernel variant (0 auto, 1 row-group register streaming, 2 bulk-copy
    ring, 3 tensor-core int4, 4 int4 register pipeline)."""
    epi = EPILOGUES[epilogue] if isinstance(epilogue, str) else int(epilogue)
    _check(lib.qne_gemv_ex(C.byref(m), _ptr(x), _ptr(y), epi, variant, ctas_per_sm, _stream(stream)))


def rmsnorm_gemv(m: _Matrix, h, norm_w, y, epilogue="store", eps: float = 1e-6, stream=None) -> None:
    epi = EPILOGUES[epilogue] if isinstance(epilogue, str) else int(epilogue)
    _check(lib.qne_rmsnorm_gemv(C.byref(m), _ptr(h), _ptr(norm_w), eps, _ptr(y), epi, _stream(stream)))


def dequant_rows(m: _Matrix, row0: int, nrows: int, out, stream=None) -> None:
    _check(lib.qne_dequant_rows(C.byref(m), row0, nrows, _ptr(out), _stream(stream)))


def embed(m: _Matrix, tok, h, stream=None) -> None:
    _check(lib.qne_embed(C.byref(m), _ptr(tok), _ptr(h), _stream(stream)))


def argmax_scratch_bytes(n: int) -> int:
    return int(lib.qne_argmax_scratch_bytes(n))


def argmax(logits, n: int, tok, scratch, scratch_bytes: int, stream=None) -> None:
    _check(lib.qne_argmax(_ptr(logits), n, _ptr(tok), _ptr(scratch), scratch_bytes, _stream(stream)))


def gdn_step(proj, conv, conv_w, state, params, counter, out, batch: int = 1, stream=None) -> None:
    _check(lib.qne_gdn_step(_ptr(proj), _ptr(conv), _ptr(conv_w), _ptr(state), _ptr(params), _ptr(counter),
                            _ptr(out), batch, _stream(stream)))


def attention_scratch_bytes(batch: int) -> int:
    return int(lib.qne_attention_scratch_bytes(batch))


ATTN_IMPLS = {"tensor_core": 0, "cuda_core": 1}


def attention_step(proj, norms, theta: float, kv, pool_pages: int, page_table, pos, out, batch, scratch,
                   scratch_bytes: int, stream=None, impl: str | None = None) -> None:
    """impl None = qne_attention_step's default kernel, else "tensor_core" or "cuda_core"."""
    if impl is None:
        _check(lib.qne_attention_step(_ptr(proj), _ptr(norms), float(theta), _ptr(kv), pool_pages, _ptr(page_table),
                                      _ptr(pos), _ptr(out), batch, _ptr(scratch), scratch_bytes, _stream(stream)))
    else:
        _check(lib.qne_attention_step_ex(_ptr(proj), _ptr(norms), float(theta), _ptr(kv), pool_pages,
                                         _ptr(page_table), _ptr(pos), _ptr(out), batch, _ptr(scratch), scratch_bytes,
                                         ATTN_IMPLS[impl], _stream(stream)))


def kv_gather(kv, page_table, length: int, out_k, out_v, stream=None) -> None:
    _check(lib.qne_kv_gather(_ptr(kv), _ptr(page_table), length, _ptr(out_k), _ptr(out_v), _stream(stream)))


def bandwidth_probe(data, nbytes: int, sink, stream=None) -> None:
    _check(lib.qne_bandwidth_probe(_ptr(data), nbytes, _ptr(sink), _stream(stream)))


DISPATCH_MODES = {"plain": 0, "graph": 1, "pdl": 2, "graph_pdl": 3}


def dispatch_cost(n: int, mode: str, y, stream=None) -> float:
    """Microseconds per launch of n noop kernels (kernels/src/lib.rs:718-724) in the given mode."""
    us = C.c_double()
    _check(lib.qne_dispatch_cost(n, DISPATCH_MODES[mode], _ptr(y), _stream(stream), C.byref(us)))
    return float(us.value)


def gemm_scratch_bytes(m: _Matrix, batch: int) -> int:
    return int(lib.qne_gemm_scratch_bytes(C.byref(m), batch))


GEMM_IMPLS = {"tcgen05": 0, "mma_sync": 1}


def gemm(m: _Matrix, x, batch: int, y, epilogue="store", scratch=None, scratch_bytes: int = 0, stream=None,
         impl: str | None = None) -> None:
    """y[batch][out_rows] (=, +=, SwiGLU) m . x[batch][k]; impl None = qne_gemm's default kernel,
    else "tcgen05" or "mma_sync" through qne_gemm_ex."""
    epi = EPILOGUES[epilogue] if isinstance(epilogue, str) else int(epilogue)
    if impl is None:
        _check(lib.qne_gemm(C.byref(m), _ptr(x), batch, _ptr(y), epi, _ptr(scratch), scratch_bytes, _stream(stream)))
    else:
        _check(lib.qne_gemm_ex(C.byref(m), _ptr(x), batch, _ptr(y), epi, GEMM_IMPLS[impl], _stream(stream)))


def _mask_words(mask):
    """Allowed-token mask (bool array, length = mask tokens) -> (uint32 words, mask tokens)."""
    if mask is None:
        return None, 0
    m = np.asarray(mask, dtype=bool)
    bits = np.zeros((m.size + 31) // 32 * 32, dtype=bool)
    bits[: m.size] = m
    words = np.packbits(bits.reshape(-1, 32)[:, ::-1], axis=1).view(">u4").astype(np.uint32).ravel()
    return np.ascontiguousarray(words), m.size


class Sampler:
    """Device-side token sampler of one generation (qne_sampler_*): the reference's
    Sampler::try_sample (src/sampling.rs) over the model's current logits or a device row."""

    def __init__(self, model: Model, temperature: float = 0.6, top_k: int = 20, top_p: float = 0.95, seed: int = 42,
                 presence_penalty: float = 0.0):
        opts = _Sampling(temperature, top_k, top_p, seed, presence_penalty)
        h = C.c_void_p()
        _check(lib.qne_sampler_create(model._h, C.byref(opts), C.byref(h)))
        self._h = h
        self.model = model
        if not hasattr(model, "_samplers"):
            model._samplers = []
        model._samplers.append(weakref.ref(self))

    def sample(self, mask=None, bias_token: int = -1, bias: float = 0.0, logits=None) -> int:
        """Draw from the model's logits, or from `logits` (a device tensor of vocab floats)."""
        words, n = _mask_words(mask)
        out = C.c_uint32()
        mp = _u32p(words) if words is not None else None
        if logits is None:
            _check(lib.qne_sampler_sample(self._h, mp, n, bias_token, float(bias), C.byref(out)))
        else:
            _check(lib.qne_sampler_sample_device(self._h, _ptr(logits), mp, n, bias_token, float(bias), C.byref(out)))
        return int(out.value)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.qne_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


if os.environ.get("QNE_PRINT_VERSION"):
    print(version())
