"""Seeded synthetic GGUF models in the shapes the decode engine is measured on.

The Local-LLM-Pure-Go engine reads its hyper-parameters from GGUF metadata
(transformer.go:1350-1421 extractConfig) and its tensors by name
(transformer.go:1122-1335 loadWeights), so a synthetic file only has to carry
those keys and tensors:

* ``{arch}.embedding_length``, ``feed_forward_length``, ``block_count``,
  ``attention.head_count[_kv]``, ``context_length``,
  ``attention.layer_norm_rms_epsilon``, ``rope.freq_base``;
* ``tokenizer.ggml.tokens`` with exactly ``vocab`` strings, because the vocab
  size is the length of that array (transformer.go:1397-1401);
* ``token_embd.weight``, ``output_norm.weight``, optional ``output.weight``
  (absent = tied embeddings), and per layer ``blk.N.{attn_q,attn_k,attn_v,
  attn_output,ffn_gate,ffn_up,ffn_down}.weight``, ``attn_norm``/``ffn_norm``
  and, for Qwen2, ``attn_{q,k,v}.bias``.

GGUF dims are ``[cols, rows]`` (dims[0] is the input width, transformer.go:1239).
Weights are N(0, 0.02) float32, norm gains 1.0, biases N(0, 0.02); 2-D weights
are quantised with the ggml rules (Q8_0: d = max|w|/127 stored as fp16,
q = roundf(w/d); Q4_0: d = w_maxabs/-8, q = min(15, trunc(w/d + 8.5)), low
nibble element j, high nibble element j+16).  Each tensor draws from its own
``SeedSequence([seed, index])`` so files are reproducible byte for byte and
written tensor by tensor without holding the model in memory.
"""
from __future__ import annotations

import dataclasses
import hashlib
import struct
from typing import Iterator

import numpy as np

GGUF_MAGIC = 0x46554747
ALIGNMENT = 32

# gguf.go:30-44 metadata value types
T_UINT32, T_INT32, T_FLOAT32, T_STRING, T_ARRAY, T_UINT64 = 4, 5, 6, 8, 9, 10
# gguf.go:47-72 tensor types
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
TYPE_NAMES = {"f32": GGML_F32, "f16": GGML_F16, "q4_0": GGML_Q4_0, "q8_0": GGML_Q8_0}
BLOCK_BYTES = {GGML_Q8_0: 34, GGML_Q4_0: 18}


@dataclasses.dataclass(frozen=True)
class ModelShape:
    arch: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    context: int
    eps: float
    theta: float
    qkv_bias: bool
    tied: bool
    wtype: str = "q8_0"
    bos_id: int = 1
    eos_id: int = 2
    # > 0: only the first distinct_layers layers have data of their own;
    # layer i's tensor infos point at the data of layer i % distinct_layers
    # (GGUF tensor infos may share offsets).  A reader still loads every
    # layer as a tensor of its own, so the bytes a decode step streams are
    # those of the full model, from a file a fraction of its size.
    distinct_layers: int = 0

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def with_(self, **kw) -> "ModelShape":
        return dataclasses.replace(self, **kw)


# The measured shapes.  Qwen2.5-0.5B: tied, QKV bias; Llama-3-8B: Q4_0, untied;
# Qwen2.5-72B: untied, QKV bias.
SHAPES = {
    "qwen2.5-0.5b": ModelShape("qwen2", 896, 24, 14, 2, 4864, 151936, 32768, 1e-6, 1e6, True, True,
                               "q8_0", 151643, 151645),
    "llama3-8b": ModelShape("llama", 4096, 32, 32, 8, 14336, 128256, 8192, 1e-5, 5e5, False, False,
                            "q4_0", 128000, 128001),
    "qwen2.5-72b": ModelShape("qwen2", 8192, 80, 64, 8, 29568, 152064, 32768, 1e-6, 1e6, True, False,
                              "q8_0", 151643, 151645),
    # Small shapes for fast oracle runs.
    "tiny": ModelShape("qwen2", 128, 2, 4, 2, 256, 512, 256, 1e-6, 1e6, True, True, "q8_0", 1, 2),
    "tiny-llama-q4": ModelShape("llama", 128, 2, 4, 1, 320, 384, 256, 1e-5, 5e5, False, False, "q4_0", 1, 2),
}
# The 72B shape cut to 4 layers (a 6.4 GB file instead of 77 GB): per-layer
# and lm_head costs of the tensor-parallel decode at the real widths.
SHAPES["qwen2.5-72b-4l"] = SHAPES["qwen2.5-72b"].with_(layers=4)
# Untied tiny model: with tied N(0, 0.02) embeddings the greedy next token is
# the input token itself, so a smoke run needs an untied head to show a
# changing greedy sequence.
SHAPES["tiny-untied"] = SHAPES["tiny"].with_(tied=False)
# Llama-3-8B widths (hidden 4096, FFN 14336, vocab 128256) cut to 4 layers:
# the config-2 parity case at its real matrix shapes.
SHAPES["llama3-8b-4l"] = SHAPES["llama3-8b"].with_(layers=4)
# Qwen2.5-72B at all 80 layers whose tensor infos share one layer's data:
# 3.6 GB on disk, 75.9 GB of weights once loaded (the tensor-parallel decode
# benchmark at the full depth).
SHAPES["qwen2.5-72b-alias"] = SHAPES["qwen2.5-72b"].with_(distinct_layers=1)


# ---------------------------------------------------------------------------
# ggml quantisation (vectorised)
# ---------------------------------------------------------------------------

def _roundf(x: np.ndarray) -> np.ndarray:
    """C roundf: halves away from zero (numpy's round is half-to-even)."""
    a = np.abs(x)
    fl = np.floor(a)
    return np.sign(x) * (fl + np.floor(2 * (a - fl)))


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """float32 [n] -> Q8_0 blocks as uint8 [n/32*34]."""
    b = np.asarray(w, dtype=np.float32).reshape(-1, 32)
    d = np.abs(b).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    qs = _roundf(b * inv).astype(np.int8)
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = qs.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """float32 [n] -> ggml Q4_0 blocks as uint8 [n/32*18]."""
    b = np.asarray(w, dtype=np.float32).reshape(-1, 32)
    imax = np.abs(b).argmax(axis=1)[:, None]
    mx = np.take_along_axis(b, imax, axis=1)
    d = mx / np.float32(-8)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np.trunc(b.astype(np.float64) * inv.astype(np.float64) + 8.5).astype(np.float32)
    q = np.clip(q.astype(np.uint8), 0, 15)
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << np.uint8(4))
    return out.reshape(-1)


def dequantize_q8_0(raw: np.ndarray, n: int) -> np.ndarray:
    blk = np.asarray(raw, dtype=np.uint8).reshape(-1, 34)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    q = blk[:, 2:].view(np.int8).astype(np.float32)
    return (d * q).reshape(-1)[:n]


def dequantize_q4_0(raw: np.ndarray, n: int) -> np.ndarray:
    """ggml layout: byte j -> element j (low nibble) and j+16 (high nibble)."""
    blk = np.asarray(raw, dtype=np.uint8).reshape(-1, 18)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    lo = (blk[:, 2:] & 0x0F).astype(np.int32) - 8
    hi = (blk[:, 2:] >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(np.float32)
    return (d * q).reshape(-1)[:n]


def quantize(w: np.ndarray, gtype: int) -> np.ndarray:
    if gtype == GGML_Q8_0:
        return quantize_q8_0(w)
    if gtype == GGML_Q4_0:
        return quantize_q4_0(w)
    if gtype == GGML_F16:
        return np.asarray(w, dtype=np.float16).view(np.uint8)
    return np.asarray(w, dtype=np.float32).view(np.uint8)


def row_bytes(gtype: int, cols: int) -> int:
    if gtype in BLOCK_BYTES:
        return cols // 32 * BLOCK_BYTES[gtype]
    return cols * (2 if gtype == GGML_F16 else 4)


# ---------------------------------------------------------------------------
# tensor plan
# ---------------------------------------------------------------------------

@dataclasses.dataclass
class TensorSpec:
    name: str
    cols: int          # dims[0]
    rows: int          # dims[1] (1 for vectors)
    gtype: int
    init: str          # "normal", "ones"
    index: int = 0
    is_vec: bool = False
    alias_of: int = -1  # index of the tensor whose data this one shares (-1: its own)

    @property
    def nbytes(self) -> int:
        return row_bytes(self.gtype, self.cols) * self.rows


def tensor_plan(shape: ModelShape) -> list[TensorSpec]:
    wt = TYPE_NAMES[shape.wtype]
    H, FF, V = shape.hidden, shape.ffn, shape.vocab
    qd, kvd = shape.heads * shape.head_dim, shape.kv_dim
    specs: list[TensorSpec] = []

    def mat(name, cols, rows, gtype=wt):
        specs.append(TensorSpec(name, cols, rows, gtype, "normal"))

    def vec(name, n, init):
        specs.append(TensorSpec(name, n, 1, GGML_F32, init, is_vec=True))

    mat("token_embd.weight", H, V)
    vec("output_norm.weight", H, "ones")
    if not shape.tied:
        mat("output.weight", H, V)
    for i in range(shape.layers):
        p = f"blk.{i}."
        vec(p + "attn_norm.weight", H, "ones")
        mat(p + "attn_q.weight", H, qd)
        mat(p + "attn_k.weight", H, kvd)
        mat(p + "attn_v.weight", H, kvd)
        if shape.qkv_bias:
            vec(p + "attn_q.bias", qd, "normal")
            vec(p + "attn_k.bias", kvd, "normal")
            vec(p + "attn_v.bias", kvd, "normal")
        mat(p + "attn_output.weight", qd, H)
        vec(p + "ffn_norm.weight", H, "ones")
        mat(p + "ffn_gate.weight", H, FF)
        mat(p + "ffn_up.weight", H, FF)
        mat(p + "ffn_down.weight", FF, H)
    for i, s in enumerate(specs):
        s.index = i
    k = shape.distinct_layers
    if k > 0:
        first = {sp.name: sp.index for sp in specs}
        for sp in specs:
            if sp.name.startswith("blk."):
                layer = int(sp.name.split(".")[1])
                if layer >= k:
                    sp.alias_of = first[sp.name.replace(f"blk.{layer}.", f"blk.{layer % k}.", 1)]
    return specs


def tensor_values(spec: TensorSpec, seed: int, chunk_rows: int | None = None) -> Iterator[np.ndarray]:
    """float32 values of a tensor, in row chunks, reproducible per tensor."""
    n_rows, cols = spec.rows, spec.cols
    if spec.init == "ones":
        yield np.ones(cols * n_rows, dtype=np.float32)
        return
    rng = np.random.default_rng(np.random.SeedSequence([seed, spec.index]))
    if chunk_rows is None:
        chunk_rows = max(1, (1 << 24) // max(cols, 1))
    for r0 in range(0, n_rows, chunk_rows):
        r = min(chunk_rows, n_rows - r0)
        yield rng.standard_normal(r * cols, dtype=np.float32) * np.float32(0.02)


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------

def _s(b: bytearray, text: str) -> None:
    e = text.encode()
    b += struct.pack("<Q", len(e)) + e


def _kv_u32(b, k, v):
    _s(b, k); b += struct.pack("<II", T_UINT32, v)


def _kv_f32(b, k, v):
    _s(b, k); b += struct.pack("<If", T_FLOAT32, v)


def _kv_str(b, k, v):
    _s(b, k); b += struct.pack("<I", T_STRING); _s(b, v)


def _kv_str_array(b, k, items):
    _s(b, k); b += struct.pack("<IIQ", T_ARRAY, T_STRING, len(items))
    for it in items:
        _s(b, it)


def _tensor_bytes(args) -> bytes:
    """All quantised bytes of one tensor (a pool worker's unit)."""
    spec, seed = args
    return b"".join(quantize(v, spec.gtype).tobytes() for v in tensor_values(spec, seed))


def write_model(path: str, shape: ModelShape, seed: int = 0, workers: int = 1, processes: bool = False) -> dict:
    """Writes a GGUF v3 file; returns {"bytes": size, "sha256": digest}.
    workers > 1 generates tensors in a thread pool (numpy's generator and
    array loops release the GIL; threads never re-import the caller's
    script), or with processes=True in a spawned process pool (faster; only
    from an import-safe main module, as this file's command line is); the
    file is identical either way, as every tensor has its own seed."""
    specs = tensor_plan(shape)
    arch = shape.arch
    meta = bytearray()
    n_kv = 0

    def count(fn, *a):
        nonlocal n_kv
        fn(meta, *a)
        n_kv += 1

    count(_kv_str, "general.architecture", arch)
    count(_kv_str, "general.name", f"synthetic-{arch}-{shape.hidden}x{shape.layers}")
    count(_kv_u32, "general.alignment", ALIGNMENT)
    count(_kv_u32, f"{arch}.context_length", shape.context)
    count(_kv_u32, f"{arch}.embedding_length", shape.hidden)
    count(_kv_u32, f"{arch}.feed_forward_length", shape.ffn)
    count(_kv_u32, f"{arch}.block_count", shape.layers)
    count(_kv_u32, f"{arch}.attention.head_count", shape.heads)
    count(_kv_u32, f"{arch}.attention.head_count_kv", shape.kv_heads)
    count(_kv_f32, f"{arch}.attention.layer_norm_rms_epsilon", shape.eps)
    count(_kv_f32, f"{arch}.rope.freq_base", shape.theta)
    count(_kv_str, "tokenizer.ggml.model", "gpt2")
    count(_kv_str_array, "tokenizer.ggml.tokens", [f"<t{i}>" for i in range(shape.vocab)])
    count(_kv_u32, "tokenizer.ggml.bos_token_id", shape.bos_id)
    count(_kv_u32, "tokenizer.ggml.eos_token_id", shape.eos_id)

    infos = bytearray()
    offset = 0
    offsets = []
    for s in specs:
        _s(infos, s.name)
        dims = (s.cols,) if s.is_vec else (s.cols, s.rows)
        infos += struct.pack("<I", len(dims))
        for d in dims:
            infos += struct.pack("<Q", d)
        own = s.alias_of < 0
        infos += struct.pack("<IQ", s.gtype, offset if own else offsets[s.alias_of])
        offsets.append(offset if own else offsets[s.alias_of])
        if own:
            offset += s.nbytes
            offset = (offset + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    data_specs = [s for s in specs if s.alias_of < 0]
    data_offsets = [offsets[s.index] for s in data_specs]

    header = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(specs), n_kv)
    h = hashlib.sha256()
    with open(path, "wb") as f:
        def w(buf):
            f.write(buf)
            h.update(buf)

        w(header)
        w(bytes(meta))
        w(bytes(infos))
        pos = len(header) + len(meta) + len(infos)
        pad = (-pos) % ALIGNMENT
        w(b"\0" * pad)
        written = 0
        pool = None
        if workers > 1:
            from concurrent.futures import ProcessPoolExecutor, ThreadPoolExecutor
            if processes:
                import multiprocessing as mp
                pool = ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn"))
            else:
                pool = ThreadPoolExecutor(workers)
            futs = [pool.submit(_tensor_bytes, (sp, seed)) for sp in data_specs]
            chunks = (f.result() for f in futs)
        else:
            chunks = (_tensor_bytes((sp, seed)) for sp in data_specs)
        try:
            for off, buf in zip(data_offsets, chunks):
                if written < off:
                    w(b"\0" * (off - written))
                    written = off
                w(buf)
                written += len(buf)
        finally:
            if pool is not None:
                pool.shutdown(wait=True, cancel_futures=True)
        tail = (-written) % ALIGNMENT
        w(b"\0" * tail)
        size = f.tell()
    return {"bytes": size, "sha256": h.hexdigest()}


def make_prompt(vocab: int, n: int, seed: int = 0) -> np.ndarray:
    """Prompt ids uniform over the vocab (the measured workloads use seed 0)."""
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


def algorithmic_bytes_per_token(shape: ModelShape) -> dict:
    """HBM bytes one B=1 decode token must read: every layer weight once, the
    lm_head blocks (token_embd when tied), the fp32 norms and biases."""
    wt = TYPE_NAMES[shape.wtype]
    H, FF, V = shape.hidden, shape.ffn, shape.vocab
    qd, kvd = shape.heads * shape.head_dim, shape.kv_dim
    layer = (row_bytes(wt, H) * (qd + 2 * kvd) + row_bytes(wt, qd) * H +
             row_bytes(wt, H) * 2 * FF + row_bytes(wt, FF) * H)
    small = 4 * (2 * H + ((qd + 2 * kvd) if shape.qkv_bias else 0))
    lm = row_bytes(wt, H) * V
    total = shape.layers * (layer + small) + lm + 4 * H
    return {"layers": shape.layers * layer, "lm_head": lm, "small": shape.layers * small + 4 * H,
            "total": total}


if __name__ == "__main__":
    # python -m b2decode.gguf_writer SHAPE OUT [--seed S] [--workers N]
    import argparse
    import os
    ap = argparse.ArgumentParser(description="write a synthetic GGUF of a named shape")
    ap.add_argument("shape", choices=sorted(SHAPES))
    ap.add_argument("out")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workers", type=int, default=os.cpu_count() or 1)
    a = ap.parse_args()
    r = write_model(a.out, SHAPES[a.shape], seed=a.seed, workers=a.workers, processes=a.workers > 1)
    print(r["bytes"], r["sha256"])
