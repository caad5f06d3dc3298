"""ctypes access to the parity oracle (libgoref.so) and the compiled reference
cross-check (_ref/libcppref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
bench's CPU-baseline leg as the checker, never by the product.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOREF_SO = os.path.join(HERE, "libgoref.so")
CPPREF_SO = os.path.join(HERE, "_ref", "libcppref.so")

MODE_GO = 0
MODE_GGML_Q4 = 1

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


class GorefConfig(C.Structure):
    _fields_ = [("arch", C.c_char * 32), ("vocab_size", C.c_int32), ("hidden_size", C.c_int32),
                ("intermediate_size", C.c_int32), ("num_layers", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("max_seq_len", C.c_int32),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("tied", C.c_int32),
                ("weight_type", C.c_int32), ("bos_id", C.c_int32), ("eos_id", C.c_int32)]


def build() -> None:
    """Compiles libgoref.so (and _ref/libcppref.so where the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(GOREF_SO):
            build()
        L = C.CDLL(GOREF_SO)
        L.goref_load.restype = C.c_void_p
        L.goref_load.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_int32]
        L.goref_free.argtypes = [C.c_void_p]
        L.goref_get_config.argtypes = [C.c_void_p, C.POINTER(GorefConfig)]
        L.goref_last_error.restype = C.c_char_p
        L.goref_reset.argtypes = [C.c_void_p]
        L.goref_cache_len.argtypes = [C.c_void_p]
        L.goref_forward.argtypes = [C.c_void_p, _i32p, C.c_int32, _f32p]
        L.goref_forward_hidden.argtypes = [C.c_void_p, _i32p, C.c_int32, _f32p]
        L.goref_argmax.argtypes = [_f32p, C.c_int32]
        L.goref_sample.argtypes = [_f32p, C.c_int32, C.c_double, C.c_int32, C.c_double, C.c_double, _i32p,
                                   C.c_int32, C.c_float]
        L.goref_predict.argtypes = [C.c_void_p, _i32p, C.c_int32, C.c_int32, C.c_double, C.c_int32, C.c_double,
                                    C.c_double, _i32p, C.c_int32, C.c_void_p, _i32p, C.POINTER(C.c_int32)]
        L.goref_dequant_tensor.restype = C.c_int64
        L.goref_dequant_tensor.argtypes = [C.c_char_p, C.c_char_p, C.c_int32, _f32p, C.c_int64]
        for fn in ("goref_matvec_q8_0", "goref_matvec_q4_0"):
            getattr(L, fn).argtypes = [_u8p, _f32p, _f32p, C.c_int32, C.c_int32]
        L.goref_matvec_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int32, C.c_int32]
        L.goref_matvec_q8_0_mt.argtypes = [C.c_void_p, _u8p, _f32p, _f32p, C.c_int32, C.c_int32]
        L.goref_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int32, C.c_int32, C.c_int32, C.c_int32]
        L.goref_rmsnorm.argtypes = [_f32p, _f32p, C.c_int32, C.c_float]
        L.goref_rope.argtypes = [_f32p, C.c_int32, C.c_int32, C.c_int32, C.c_float]
        L.goref_silu.restype = C.c_float
        L.goref_silu.argtypes = [C.c_float]
        L.goref_softmax.argtypes = [_f32p, C.c_int32]
        L.goref_f16_to_f32.restype = C.c_float
        L.goref_f16_to_f32.argtypes = [C.c_uint16]
        L.goref_pool_only.restype = C.c_void_p
        L.goref_pool_only.argtypes = [C.c_int32]
        L.goref_num_threads.argtypes = [C.c_void_p]
        _lib = L
    return _lib


class GoRef:
    """The Go engine restated: load a GGUF, run forward / predict."""

    def __init__(self, path: str, num_ctx: int = 0, n_threads: int = 0, mode: int = MODE_GO):
        L = lib()
        self._h = L.goref_load(path.encode(), num_ctx, n_threads, mode)
        if not self._h:
            raise RuntimeError("goref_load: " + L.goref_last_error().decode())
        c = GorefConfig()
        L.goref_get_config(self._h, C.byref(c))
        self.cfg = {k: getattr(c, k) for k, _ in GorefConfig._fields_}
        self.cfg["arch"] = c.arch.decode()
        self.vocab = c.vocab_size

    def close(self):
        if self._h:
            lib().goref_free(self._h)
            self._h = None

    __del__ = close

    def reset(self):
        lib().goref_reset(self._h)

    @property
    def cache_len(self) -> int:
        return lib().goref_cache_len(self._h)

    @property
    def threads(self) -> int:
        return lib().goref_num_threads(self._h)

    def forward(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float32)
        if lib().goref_forward(self._h, t, len(t), out) != 0:
            raise RuntimeError("goref_forward: " + lib().goref_last_error().decode())
        return out

    def forward_hidden(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.cfg["hidden_size"], dtype=np.float32)
        if lib().goref_forward_hidden(self._h, t, len(t), out) != 0:
            raise RuntimeError("goref_forward_hidden failed")
        return out

    def predict(self, prompt, max_gen, temperature=0.001, top_k=0, top_p=0.0, repeat_penalty=1.0,
                stop_ids=(), uniforms=None) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        s = np.ascontiguousarray(stop_ids, dtype=np.int32).reshape(-1)
        if s.size == 0:
            s = np.zeros(1, dtype=np.int32)
            n_stop = 0
        else:
            n_stop = s.size
        u = None
        if uniforms is not None:
            u_arr = np.ascontiguousarray(uniforms, dtype=np.float32)
            u = u_arr.ctypes.data_as(C.c_void_p)
        out = np.zeros(max(max_gen, 256) if max_gen <= 0 else max_gen, dtype=np.int32)
        n = C.c_int32(0)
        rc = lib().goref_predict(self._h, p, len(p), max_gen, temperature, top_k, top_p, repeat_penalty, s,
                                 n_stop, u, out, C.byref(n))
        if rc != 0:
            raise RuntimeError("goref_predict: " + lib().goref_last_error().decode())
        return out[: n.value].copy()


def dequant_tensor(path: str, name: str, n: int, mode: int = MODE_GO) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    got = lib().goref_dequant_tensor(path.encode(), name.encode(), mode, out, n)
    if got < 0:
        raise RuntimeError(lib().goref_last_error().decode())
    return out[:got]


def matvec(kind: str, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if kind == "q8_0":
        lib().goref_matvec_q8_0(np.ascontiguousarray(w, dtype=np.uint8), x, y, rows, cols)
    elif kind == "q4_0":
        lib().goref_matvec_q4_0(np.ascontiguousarray(w, dtype=np.uint8), x, y, rows, cols)
    else:
        lib().goref_matvec_f32(np.ascontiguousarray(w, dtype=np.float32), x, y, rows, cols)
    return y


def attention(q, k, v, nh, nkv, hd, ctx) -> np.ndarray:
    out = np.empty(nh * hd, dtype=np.float32)
    lib().goref_attention(np.ascontiguousarray(q, dtype=np.float32), np.ascontiguousarray(k, dtype=np.float32),
                          np.ascontiguousarray(v, dtype=np.float32), out, nh, nkv, hd, ctx)
    return out


def sample(logits, temperature, top_k, top_p, repeat_penalty, generated, r) -> int:
    lg = np.array(logits, dtype=np.float32, copy=True)
    g = np.ascontiguousarray(generated, dtype=np.int32).reshape(-1)
    if g.size == 0:
        g = np.zeros(1, dtype=np.int32)
        ng = 0
    else:
        ng = g.size
    return int(lib().goref_sample(lg, lg.size, temperature, top_k, top_p, repeat_penalty, g, ng, r))


# ---------------------------------------------------------------------------
# compiled reference (C++ sibling engine)
# ---------------------------------------------------------------------------

_cpp = None


def cppref_available() -> bool:
    return os.path.exists(CPPREF_SO)


def cpplib():
    global _cpp
    if _cpp is None:
        L = C.CDLL(CPPREF_SO)
        L.cppref_load.restype = C.c_void_p
        L.cppref_load.argtypes = [C.c_char_p]
        L.cppref_free.argtypes = [C.c_void_p]
        L.cppref_vocab.argtypes = [C.c_void_p]
        L.cppref_reset.argtypes = [C.c_void_p]
        L.cppref_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, C.c_int]
        L.cppref_dequant_q4_0.argtypes = [_u8p, _f32p, C.c_longlong]
        L.cppref_dequant_q8_0.argtypes = [_u8p, _f32p, C.c_longlong]
        L.cppref_vec_dot_q8_0.restype = C.c_float
        L.cppref_vec_dot_q8_0.argtypes = [_u8p, _f32p, C.c_longlong]
        L.cppref_vec_dot_q4_0.restype = C.c_float
        L.cppref_vec_dot_q4_0.argtypes = [_u8p, _f32p, C.c_longlong]
        _cpp = L
    return _cpp


class CppRef:
    """The reference's C++ sibling engine, driven token by token."""

    def __init__(self, path: str):
        L = cpplib()
        self._h = L.cppref_load(path.encode())
        if not self._h:
            raise RuntimeError("cppref_load failed")
        self.vocab = L.cppref_vocab(self._h)
        self.pos = 0

    def close(self):
        if self._h:
            cpplib().cppref_free(self._h)
            self._h = None

    __del__ = close

    def reset(self):
        cpplib().cppref_reset(self._h)
        self.pos = 0

    def forward(self, tokens) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        for t in tokens:
            cpplib().cppref_forward(self._h, int(t), self.pos, out, self.vocab)
            self.pos += 1
        return out


def cppref_dequant(kind: str, raw: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    fn = cpplib().cppref_dequant_q4_0 if kind == "q4_0" else cpplib().cppref_dequant_q8_0
    fn(np.ascontiguousarray(raw, dtype=np.uint8), out, n)
    return out
