"""Python access to the b2decode C ABI (include/b2decode.h).

The library is the product; this module only binds it with ctypes for tests,
the smoke check and the bench.  It refuses to run without the compiled
library: there is no Python or CPU fallback for any computation.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Iterator, Sequence

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libb2decode.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "b2decode.h")

B2_OK = 0
TRACE_SLOTS = 13  # slots per phase and CTA in trace_step (kTraceSlots)
PHASES_PER_LAYER = 4  # decode phases per layer (kPhasesPerLayer)
ERRORS = {
    -1: "IO", -2: "FORMAT", -3: "UNSUPPORTED_TYPE", -4: "OOM", -5: "CUDA", -6: "NCCL", -7: "TIMEOUT",
    -8: "BAD_ARG", -9: "CONTEXT", -10: "NOT_LOADED",
}
QTYPE_Q8_0 = 8
QTYPE_Q4_0 = 2


class TpShare(C.Structure):
    _fields_ = [("q_row0", C.c_int32), ("q_rows", C.c_int32), ("kv_row0", C.c_int32), ("kv_rows", C.c_int32),
                ("ffn_row0", C.c_int32), ("ffn_rows", C.c_int32), ("vocab_row0", C.c_int32),
                ("vocab_rows", C.c_int32)]


class B2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"B2_ERR_{ERRORS.get(code, code)} ({code}): {msg}")
        self.code = code


class LoadOpts(C.Structure):
    _fields_ = [("num_ctx", C.c_int32), ("device", C.c_int32), ("kv_fp32", C.c_int32), ("tp_size", C.c_int32),
                ("tp_rank", C.c_int32), ("reserved2", C.c_int32)]


class LoadStats(C.Structure):
    _fields_ = [("total_ns", C.c_int64), ("parse_ns", C.c_int64), ("upload_ns", C.c_int64),
                ("host_copy_ns", C.c_int64), ("bytes_uploaded", C.c_int64), ("host_threads", C.c_int32),
                ("mapped", C.c_int32), ("setup_ns", C.c_int64)]


class Config(C.Structure):
    _fields_ = [("arch", C.c_char * 32), ("vocab_size", C.c_int32), ("hidden_size", C.c_int32),
                ("intermediate_size", C.c_int32), ("num_layers", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("max_seq_len", C.c_int32),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("tied_embeddings", C.c_int32),
                ("has_qkv_bias", C.c_int32), ("weight_type", C.c_int32), ("bos_id", C.c_int32),
                ("eos_id", C.c_int32), ("weight_bytes", C.c_int64), ("stream_bytes_per_token", C.c_int64),
                ("tp_size", C.c_int32), ("tp_rank", C.c_int32), ("vocab_begin", C.c_int32), ("vocab_local", C.c_int32)]


class Timings(C.Structure):
    _fields_ = [("prompt_ns", C.c_int64), ("eval_ns", C.c_int64), ("prompt_tokens", C.c_int32),
                ("completion_tokens", C.c_int32)]


class SampleOpts(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_k", C.c_int32), ("top_p", C.c_double),
                ("repeat_penalty", C.c_double), ("num_predict", C.c_int32), ("seed", C.c_uint64)]


def build(verbose: bool = False) -> str:
    """Compiles libb2decode.so in-tree (nvcc, sm_100a)."""
    out = subprocess.run(["make", "-j8", "-C", PKG_DIR], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("libb2decode build failed:\n" + out.stdout[-4000:] + out.stderr[-4000:])
    if verbose:
        print(out.stdout[-2000:])
    return LIB_PATH


_lib = None

_P = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_i32p = C.POINTER(C.c_int32)
_f32p = C.POINTER(C.c_float)

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "b2_load": (C.c_int, [C.c_char_p, C.POINTER(LoadOpts), C.POINTER(_P)]),
    "b2_free": (None, [_P]),
    "b2_get_config": (C.c_int, [_P, C.POINTER(Config)]),
    "b2_get_load_stats": (C.c_int, [_P, C.POINTER(LoadStats)]),
    "b2_last_error": (C.c_char_p, []),
    "b2_reset": (C.c_int, [_P]),
    "b2_cache_len": (C.c_int, [_P, _i32p]),
    "b2_forward": (C.c_int, [_P, _i32p, _i32, _f32p]),
    "b2_forward_argmax": (C.c_int, [_P, _i32p, _i32, _i32p]),
    "b2_decode_greedy": (C.c_int, [_P, _i32, _i32, _i32, _i32p, _i32p]),
    "b2_predict": (C.c_int, [_P, _i32p, _i32, C.POINTER(SampleOpts), _i32p, _i32, _i32p, _i32, _i32p,
                             C.POINTER(Timings)]),
    "b2_stream_begin": (C.c_int, [_P, _i32p, _i32, C.POINTER(SampleOpts), _i32p, _i32]),
    "b2_stream_next": (C.c_int, [_P, _i32p, _i32p]),
    "b2_sample_logits": (C.c_int32, [_f32p, _i32, C.POINTER(SampleOpts), _i32p, _i32, C.c_float]),
    "b2_sample_device": (C.c_int, [_P, _i32, _i32, _i64, C.POINTER(SampleOpts), _P, _i64, _i32p, _f32p, _P, _P, _P]),
    "b2_sample_scratch_bytes": (_i64, [_i32, _i32]),
    "b2_embed": (C.c_int, [_P, _i32p, _i32, _f32p]),
    "b2_dequant_tensor": (C.c_int, [_P, C.c_char_p, _f32p, _i64, C.POINTER(_i64)]),
    "b2_matvec": (C.c_int, [_i32, _P, _P, _P, _i32, _i32, _P]),
    "b2_matvec_batch": (C.c_int, [_i32, _P, _P, _P, _i32, _i32, _i32, _P]),
    "b2_model_matvec": (C.c_int, [_P, C.c_char_p, _P, _P, _i32, _P]),
    "b2_model_gemm": (C.c_int, [_P, C.c_char_p, _P, _P, _i32, _P]),
    "b2_batch_create": (C.c_int, [_P, _i32, C.POINTER(_P)]),
    "b2_batch_free": (None, [_P]),
    "b2_batch_prefill": (C.c_int, [_P, _i32, _i32p, _i32, C.POINTER(_i32)]),
    "b2_batch_step": (C.c_int, [_P, _i32p, _i32p]),
    "b2_batch_logits": (C.c_int, [_P, _f32p]),
    "b2_batch_use_graph": (C.c_int, [_P, _i32]),
    "b2_attention_decode": (C.c_int, [_P, _P, _P, _P, _i32, _i32, _i32, _i32, _i32, _P]),
    "b2_attention_decode_noalloc": (C.c_int, [_P, _P, _P, _P, _i32, _i32, _i32, _i32, _i32, _P]),
    "b2_device_status": (C.c_int, [_P]),
    "b2_stream_handle": (_P, [_P]),
    "b2_trace_step": (C.c_int, [_P, _i32, C.POINTER(_i64), _i64, _i32p, _i32p]),
    "b2_debug_wait_skew": (C.c_int, [_P, _i32]),
    "b2_debug_fail_alloc": (C.c_int, [_i32]),
    "b2_tp_share_of": (C.c_int, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, C.POINTER(TpShare)]),
    "b2_tp_handle": (C.c_int, [_P, C.c_char_p]),
    "b2_tp_connect": (C.c_int, [_P, C.c_char_p]),
}


def lib():
    """Loads libb2decode.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it first (make -C {PKG_DIR}); "
                               "there is no fallback implementation")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().b2_last_error().decode(errors="replace")


def _check(rc: int) -> None:
    if rc != B2_OK:
        raise B2Error(rc, last_error())


def _ids(a) -> tuple:
    arr = np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))
    return arr, arr.ctypes.data_as(_i32p)


def sample_opts(temperature=0.0, top_k=0, top_p=0.0, repeat_penalty=1.0, num_predict=0, seed=0) -> SampleOpts:
    return SampleOpts(float(temperature), int(top_k), float(top_p), float(repeat_penalty), int(num_predict),
                      int(seed))


class Model:
    """One loaded GGUF model on one GPU (a b2_model handle).  With tp_size > 1
    it is rank tp_rank's share of a tensor-parallel model: connect all ranks
    (tp.connect) before the first forward call."""

    def __init__(self, path: str, num_ctx: int = 0, device: int = 0, kv_fp32: bool = False, tp_size: int = 1,
                 tp_rank: int = 0):
        L = lib()
        opts = LoadOpts(int(num_ctx), int(device), 1 if kv_fp32 else 0, int(tp_size), int(tp_rank), 0)
        h = _P()
        _check(L.b2_load(path.encode(), C.byref(opts), C.byref(h)))
        self._h = h
        c = Config()
        _check(L.b2_get_config(self._h, C.byref(c)))
        self.cfg = {k: getattr(c, k) for k, _ in Config._fields_}
        self.cfg["arch"] = c.arch.decode()
        self.vocab = c.vocab_size

    def load_stats(self) -> dict:
        """b2_get_load_stats: where the load's time went."""
        s = LoadStats()
        _check(lib().b2_get_load_stats(self._h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in LoadStats._fields_}

    def tp_handle(self) -> bytes:
        """64-byte IPC handle of this rank's exchange buffer."""
        buf = C.create_string_buffer(64)
        _check(lib().b2_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles) -> None:
        """Maps every rank's exchange buffer (handles in rank order)."""
        blob = b"".join(bytes(h) for h in handles)
        if len(blob) != 64 * len(handles):
            raise ValueError("handles must be 64 bytes each")
        _check(lib().b2_tp_connect(self._h, blob))

    # engine.go Unload
    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().b2_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def reset(self) -> None:
        _check(lib().b2_reset(self._h))

    @property
    def cache_len(self) -> int:
        n = C.c_int32()
        _check(lib().b2_cache_len(self._h, C.byref(n)))
        return n.value

    def forward(self, tokens) -> np.ndarray:
        """Logits of the last token: the whole vocabulary, or this rank's share
        (cfg vocab_begin .. + vocab_local) of a tensor-parallel model."""
        arr, p = _ids(tokens)
        out = np.empty(self.cfg["vocab_local"], dtype=np.float32)
        _check(lib().b2_forward(self._h, p, len(arr), out.ctypes.data_as(_f32p)))
        return out

    def forward_argmax(self, tokens) -> int:
        arr, p = _ids(tokens)
        nxt = C.c_int32()
        _check(lib().b2_forward_argmax(self._h, p, len(arr), C.byref(nxt)))
        return nxt.value

    def decode_greedy(self, first: int, n_steps: int, eos: int = -1) -> np.ndarray:
        out = np.zeros(max(n_steps, 1), dtype=np.int32)
        n = C.c_int32()
        _check(lib().b2_decode_greedy(self._h, int(first), int(n_steps), int(eos), out.ctypes.data_as(_i32p),
                                      C.byref(n)))
        return out[: n.value].copy()

    def predict(self, prompt, opts: SampleOpts | None = None, stop_ids: Sequence[int] = (), max_out: int = 4096):
        arr, p = _ids(prompt)
        st, sp = _ids(list(stop_ids) or [0])
        out = np.zeros(max_out, dtype=np.int32)
        n = C.c_int32()
        t = Timings()
        _check(lib().b2_predict(self._h, p, len(arr), C.byref(opts or sample_opts()), sp, len(stop_ids),
                                out.ctypes.data_as(_i32p), max_out, C.byref(n), C.byref(t)))
        return out[: n.value].copy(), {k: getattr(t, k) for k, _ in Timings._fields_}

    def stream(self, prompt, opts: SampleOpts | None = None, stop_ids: Sequence[int] = ()) -> Iterator[int]:
        arr, p = _ids(prompt)
        st, sp = _ids(list(stop_ids) or [0])
        _check(lib().b2_stream_begin(self._h, p, len(arr), C.byref(opts or sample_opts()), sp, len(stop_ids)))
        tok, done = C.c_int32(), C.c_int32()
        while True:
            _check(lib().b2_stream_next(self._h, C.byref(tok), C.byref(done)))
            if done.value:
                return
            yield tok.value

    def embed(self, tokens) -> np.ndarray:
        arr, p = _ids(tokens)
        out = np.empty(self.cfg["hidden_size"], dtype=np.float32)
        _check(lib().b2_embed(self._h, p, len(arr), out.ctypes.data_as(_f32p)))
        return out

    def dequant(self, name: str, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        got = C.c_int64()
        _check(lib().b2_dequant_tensor(self._h, name.encode(), out.ctypes.data_as(_f32p), n, C.byref(got)))
        return out[: got.value]

    def matvec(self, name: str, x_ptr: int, y_ptr: int, nvec: int, stream: int = 0) -> None:
        """Y = W X over the resident tensor `name` for nvec (1..16) vectors:
        x [nvec][cols], y [nvec][rows] fp32 at device addresses."""
        _check(lib().b2_model_matvec(self._h, name.encode(), x_ptr, y_ptr, nvec, stream or None))

    def gemm(self, name: str, x_ptr: int, y_ptr: int, ntok: int, stream: int = 0) -> None:
        """Y = W X over the resident tensor `name` for ntok tokens on the tensor
        cores: x [ntok][cols], y [ntok][rows] fp32 at device addresses."""
        _check(lib().b2_model_gemm(self._h, name.encode(), x_ptr, y_ptr, ntok, stream or None))

    def device_status(self) -> int:
        return lib().b2_device_status(self._h)

    def trace_step(self, token: int) -> np.ndarray:
        """[phases, TRACE_SLOTS, ctas] timeline of one decode step: globaltimer
        stamps (ns) in slots 0-5, consumer chunk-wait ns and slow-wait count in
        6-7, producer slot-wait ns and chunks issued in 8-9, rows loop done in 10,
        ns in tile dot products in 11, epilogue constants ready in 12."""
        P = PHASES_PER_LAYER * self.cfg["num_layers"] + 1
        cap = P * TRACE_SLOTS * 1024
        out = np.zeros(cap, dtype=np.int64)
        npz, nc = C.c_int32(), C.c_int32()
        _check(lib().b2_trace_step(self._h, int(token), out.ctypes.data_as(C.POINTER(_i64)), cap, C.byref(npz),
                                   C.byref(nc)))
        return out[: npz.value * TRACE_SLOTS * nc.value].reshape(npz.value, TRACE_SLOTS, nc.value)

    def stream_handle(self) -> int:
        return lib().b2_stream_handle(self._h) or 0

    def debug_wait_skew(self, skew: int) -> None:
        _check(lib().b2_debug_wait_skew(self._h, int(skew)))


def tp_share_of(hidden: int, heads: int, kv_heads: int, ffn: int, vocab: int, tp: int, rank: int) -> dict:
    """The slices a tensor-parallel rank keeps, computed by the loader's own
    arithmetic (b2_tp_share_of; host only): (first, end) ranges."""
    s = TpShare()
    _check(lib().b2_tp_share_of(hidden, heads, kv_heads, ffn, vocab, tp, rank, C.byref(s)))
    q = (s.q_row0, s.q_row0 + s.q_rows)
    f = (s.ffn_row0, s.ffn_row0 + s.ffn_rows)
    return {"q_rows": q, "kv_rows": (s.kv_row0, s.kv_row0 + s.kv_rows), "wo_cols": q, "ffn_rows": f,
            "down_cols": f, "vocab_rows": (s.vocab_row0, s.vocab_row0 + s.vocab_rows)}


def debug_fail_alloc(nth: int) -> None:
    """The nth device allocation of the next loads fails (b2_debug_fail_alloc); 0 disarms."""
    _check(lib().b2_debug_fail_alloc(int(nth)))


def sample_logits(logits, opts: SampleOpts, generated=(), r: float = 0.5) -> int:
    lg = np.array(logits, dtype=np.float32, copy=True)
    g, gp = _ids(list(generated) or [0])
    return int(lib().b2_sample_logits(lg.ctypes.data_as(_f32p), lg.size, C.byref(opts), gp, len(generated),
                                      float(r)))


def sample_scratch_bytes(n: int, rows: int) -> int:
    """Device scratch b2_sample_device needs for rows rows of n logits."""
    return int(lib().b2_sample_scratch_bytes(n, rows))


def sample_device(d_logits: int, n: int, rows: int, ld: int, opts: SampleOpts, d_generated: int = 0,
                  gen_ld: int = 0, n_generated=None, r=(0.5,), d_scratch: int = 0, d_out: int = 0,
                  stream: int = 0) -> None:
    """b2_sample_device on device pointers (logits modified in place; d_scratch
    of sample_scratch_bytes(n, rows) bytes); the ids land in d_out[rows] on
    `stream`."""
    ng = (C.c_int32 * rows)(*(list(n_generated) if n_generated is not None else [0] * rows))
    rr = (C.c_float * rows)(*[float(x) for x in r])
    _check(lib().b2_sample_device(d_logits, n, rows, ld, C.byref(opts), d_generated or None, gen_ld,
                                  C.cast(ng, _i32p), C.cast(rr, _f32p), d_scratch or None, d_out, stream or None))


class Batch:
    """Batched greedy decode over a loaded single-GPU Model: `batch` slots,
    each a sequence with its own KV cache, advancing one token per step
    together (b2_batch_*)."""

    def __init__(self, model: "Model", batch: int):
        h = _P()
        _check(lib().b2_batch_create(model._h, int(batch), C.byref(h)))
        self._h, self.model, self.batch = h, model, int(batch)
        self.vocab = int(model.vocab)

    def prefill(self, slot: int, prompt) -> int:
        """Runs the prompt into the slot; returns the argmax after it."""
        arr, p = _ids(prompt)
        nxt = C.c_int32()
        _check(lib().b2_batch_prefill(self._h, int(slot), p, len(arr), C.byref(nxt)))
        return nxt.value

    def step(self, tokens) -> np.ndarray:
        """Feeds one token per slot; returns the next id of every slot."""
        arr, p = _ids(tokens)
        if len(arr) != self.batch:
            raise ValueError("one token per slot")
        out = np.zeros(self.batch, dtype=np.int32)
        _check(lib().b2_batch_step(self._h, p, out.ctypes.data_as(_i32p)))
        return out

    def use_graph(self, on: bool = True) -> None:
        """Replay steps from a captured CUDA graph (b2_batch_use_graph)."""
        _check(lib().b2_batch_use_graph(self._h, 1 if on else 0))

    def logits(self) -> np.ndarray:
        out = np.empty((self.batch, self.vocab), dtype=np.float32)
        _check(lib().b2_batch_logits(self._h, out.ctypes.data_as(_f32p)))
        return out

    def close(self) -> None:
        if self._h:
            lib().b2_batch_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def matvec(qtype: int, w_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, stream: int = 0) -> None:
    """y = W x on the device; pointers are device addresses (e.g. tensor.data_ptr())."""
    _check(lib().b2_matvec(qtype, w_ptr, x_ptr, y_ptr, rows, cols, stream or None))


def matvec_batch(qtype: int, w_ptr: int, x_ptr: int, y_ptr: int, rows: int, cols: int, nvec: int,
                 stream: int = 0) -> None:
    """Y = W X for nvec (1..16) vectors in one pass over W: x [nvec][cols], y [nvec][rows] fp32, device addresses."""
    _check(lib().b2_matvec_batch(qtype, w_ptr, x_ptr, y_ptr, rows, cols, nvec, stream or None))


def attention_decode(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, batch: int, nh: int, nkv: int, hd: int,
                     ctx: int, stream: int = 0) -> None:
    _check(lib().b2_attention_decode(q_ptr, k_ptr, v_ptr, out_ptr, batch, nh, nkv, hd, ctx, stream or None))


def attention_decode_noalloc(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, batch: int, nh: int, nkv: int,
                             hd: int, ctx: int, stream: int = 0) -> None:
    """attention_decode without device allocation (fixed in-library scratch)."""
    _check(lib().b2_attention_decode_noalloc(q_ptr, k_ptr, v_ptr, out_ptr, batch, nh, nkv, hd, ctx, stream or None))
