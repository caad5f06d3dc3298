"""The C ABI without a GPU: the library loads, exports every symbol the
header declares, rejects malformed GGUF files with the right error codes and
samples host logits exactly as the Go engine's sample() does."""
import os
import re
import struct

import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw
from conftest import has_gpu

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "b2decode.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(b2_[a-z_0-9]+)\s*\(", src)))


def test_header_symbols_exported(built_lib):
    names = declared_symbols()
    assert len(names) >= 18
    for n in names:
        assert hasattr(built_lib, n), n
    assert set(names) == set(b2decode.SIGNATURES), set(names) ^ set(b2decode.SIGNATURES)


def test_library_is_sm100a(built_lib):
    out = os.popen(f"cuobjdump --list-elf {b2decode.LIB_PATH} 2>/dev/null").read()
    if out:
        assert "sm_100a" in out


def _load_err(path):
    try:
        b2decode.Model(path)
    except b2decode.B2Error as e:
        return e.code, str(e)
    return 0, ""


def test_missing_file(built_lib, tmp_path):
    code, msg = _load_err(str(tmp_path / "nope.gguf"))
    assert code == -1 and "open" in msg


def test_bad_magic_and_version(built_lib, tmp_path, tiny_gguf):
    raw = bytearray(open(tiny_gguf, "rb").read())
    p = tmp_path / "badmagic.gguf"
    bad = bytearray(raw)
    bad[0:4] = b"GGUX"
    p.write_bytes(bad)
    code, msg = _load_err(str(p))
    assert code == -2 and "magic" in msg
    bad = bytearray(raw)
    bad[4:8] = struct.pack("<I", 7)
    p.write_bytes(bad)
    code, msg = _load_err(str(p))
    assert code == -2 and "version" in msg


def test_truncated_file(built_lib, tmp_path, tiny_gguf):
    raw = open(tiny_gguf, "rb").read()
    for cut in (10, 200, len(raw) - 4096):
        p = tmp_path / f"trunc{cut}.gguf"
        p.write_bytes(raw[:cut])
        code, _ = _load_err(str(p))
        assert code == -2, cut


def test_unsupported_weight_type(built_lib, tmp_path):
    shape = gw.SHAPES["tiny"].with_(wtype="f16")
    p = str(tmp_path / "f16.gguf")
    gw.write_model(p, shape)
    code, msg = _load_err(p)
    assert code == -3, msg


@pytest.mark.skipif(has_gpu(), reason="checks the no-GPU error path")
def test_no_gpu_is_an_error_not_a_fallback(built_lib, tiny_gguf):
    code, msg = _load_err(tiny_gguf)
    assert code == -5 and "no CUDA device" in msg


def test_null_handles(built_lib):
    L = built_lib
    assert L.b2_reset(None) == -10
    assert L.b2_forward(None, None, 0, None) == -10
    L.b2_free(None)


@pytest.mark.parametrize("seed", range(6))
def test_host_sampler_matches_go_sample(built_lib, oracle_lib, seed):
    rng = np.random.default_rng(seed)
    V = 4096
    lg = (rng.standard_normal(V) * 3).astype(np.float32)
    gen = rng.integers(0, V, 20).tolist()
    cases = [(0.001, 0, 0.0, 1.0), (0.001, 0, 0.0, 1.3), (0.7, 40, 0.9, 1.1), (1.0, 0, 0.0, 1.0),
             (0.0, 0, 0.95, 1.0), (0.8, 5, 0.0, 1.0), (1.5, 0, 0.5, 2.0)]
    for temp, k, p, rp in cases:
        for r in (0.0, 0.1234, 0.5, 0.987):
            want = goref.sample(lg, temp, k, p, rp, gen, r)
            got = b2decode.sample_logits(lg, b2decode.sample_opts(temp, k, p, rp), gen, r)
            assert got == want, (temp, k, p, rp, r)


def _tp_load_err(path, tp_size, tp_rank):
    try:
        b2decode.Model(path, tp_size=tp_size, tp_rank=tp_rank)
    except b2decode.B2Error as e:
        return e.code, str(e)
    return 0, ""


def test_tensor_parallel_options_checked_before_any_device_work(built_lib, tiny_gguf):
    # degree above 8, rank outside the degree: bad arguments
    assert _tp_load_err(tiny_gguf, 9, 0)[0] == -8
    assert _tp_load_err(tiny_gguf, 2, 2)[0] == -8
    assert _tp_load_err(tiny_gguf, 2, -1)[0] == -8
    # the tiny model has 2 KV heads: 4 ranks cannot share them
    code, msg = _tp_load_err(tiny_gguf, 4, 1)
    assert code == -3 and "divisible" in msg


@pytest.mark.skipif(has_gpu(), reason="the CPU-only path")
def test_tensor_parallel_load_needs_a_gpu(built_lib, tiny_gguf):
    code, msg = _tp_load_err(tiny_gguf, 2, 1)
    assert code == -5 and "no CUDA device" in msg


def test_model_matvec_rejects_null_model(built_lib):
    assert b2decode.lib().b2_model_matvec(None, b"token_embd.weight", 4096, 8192, 8, None) == -10


def test_batch_entry_points_reject_null(built_lib):
    L = b2decode.lib()
    h = b2decode._P()
    assert L.b2_batch_create(None, 4, b2decode.C.byref(h)) == -10
    toks = (b2decode.C.c_int32 * 4)()
    assert L.b2_batch_step(None, toks, toks) == -10
    assert L.b2_batch_prefill(None, 0, toks, 4, toks) == -10
    assert L.b2_batch_logits(None, None) == -10
    L.b2_batch_free(None)


def test_tp_entry_points_reject_null(built_lib):
    L = b2decode.lib()
    assert L.b2_tp_handle(None, b"\0" * 64) == -10
    assert L.b2_tp_connect(None, b"\0" * 64) == -10


@pytest.mark.parametrize("qtype,rows,cols,nvec,code,text", [
    (8, 64, 4096, 0, -8, "1 to 16 vectors"),
    (8, 64, 4096, 17, -8, "1 to 16 vectors"),
    (8, 64, 4000, 8, -8, "multiple of 256"),
    (2, 64, 288, 8, -8, "multiple of 256"),
    (8, 0, 4096, 8, -8, "bad matvec arguments"),
    (3, 64, 4096, 8, -3, "qtype"),
])
def test_batched_matvec_arguments_checked_before_any_device_work(built_lib, qtype, rows, cols, nvec, code, text):
    """Bad shapes are rejected by the C ABI itself: the (never dereferenced)
    device addresses below would fault if any of these reached a kernel."""
    L = b2decode.lib()
    assert L.b2_matvec_batch(qtype, 4096, 8192, 16384, rows, cols, nvec, None) == code
    assert text in b2decode.last_error()
    assert L.b2_matvec_batch(8, None, 8192, 16384, 64, 4096, 8, None) == -8


def test_batched_matvec_alignment_and_no_gpu(built_lib):
    L = b2decode.lib()
    assert L.b2_matvec_batch(8, 4100, 8192, 16384, 64, 4096, 8, None) == -8
    assert "16-byte aligned" in b2decode.last_error()
    if not has_gpu():
        assert L.b2_matvec_batch(8, 4096, 8192, 16384, 64, 4096, 8, None) == -5
        assert "no CUDA device" in b2decode.last_error()
