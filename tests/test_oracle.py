"""The oracle pinned: goref (CPU restatement of the Go engine) against the
ggml quantisation rules of gguf-py, the committed golden fixtures and the
reference's compiled C++ sibling engine."""
import json
import os

import numpy as np
import pytest

import goref
from b2decode import gguf_writer as gw

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_quantizers_match_gguf_py():
    from gguf import GGMLQuantizationType as Q, quants
    rng = np.random.default_rng(3)
    w = rng.standard_normal(32 * 512, dtype=np.float32) * 0.02
    w[:32] = 0.0
    w[32:64] = 1e-8
    for q, fn in ((Q.Q8_0, gw.quantize_q8_0), (Q.Q4_0, gw.quantize_q4_0)):
        ref = quants.quantize(w.reshape(16, -1), q).reshape(-1)
        assert np.array_equal(fn(w), ref)
        assert np.array_equal(quants.dequantize(ref.reshape(16, -1), q).reshape(-1),
                              gw.dequantize_q8_0(ref, w.size) if q == Q.Q8_0 else gw.dequantize_q4_0(ref, w.size))


def test_writer_is_pinned(tiny_gguf, tiny_q4_gguf):
    import hashlib
    for path, key in ((tiny_gguf, "tiny"), (tiny_q4_gguf, "tiny-llama-q4")):
        assert hashlib.sha256(open(path, "rb").read()).hexdigest() == GOLDEN[key]["sha256"]


def test_f16_all_bit_patterns(oracle_lib):
    L = goref.lib()
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([L.goref_f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))


def test_dequant_q8_bit_exact(oracle_lib, tiny_gguf):
    from gguf import GGUFReader
    r = GGUFReader(tiny_gguf)
    t = next(t for t in r.tensors if t.name == "blk.0.attn_q.weight")
    n = int(t.n_elements)
    ref = gw.dequantize_q8_0(np.asarray(t.data).reshape(-1).view(np.uint8), n)
    got = goref.dequant_tensor(tiny_gguf, "blk.0.attn_q.weight", n)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_q4_orders(oracle_lib, tiny_q4_gguf):
    from gguf import GGUFReader, GGMLQuantizationType as Q, quants
    r = GGUFReader(tiny_q4_gguf)
    t = next(t for t in r.tensors if t.name == "blk.0.ffn_up.weight")
    n = int(t.n_elements)
    raw = np.asarray(t.data).reshape(-1).view(np.uint8)
    ggml = quants.dequantize(raw.reshape(-1, 18), Q.Q4_0).reshape(-1)
    got = goref.dequant_tensor(tiny_q4_gguf, "blk.0.ffn_up.weight", n, mode=goref.MODE_GGML_Q4)
    assert np.array_equal(got, ggml)
    # gguf.go:598-609 puts nibbles of byte j at elements 2j, 2j+1: a different order
    go = goref.dequant_tensor(tiny_q4_gguf, "blk.0.ffn_up.weight", n, mode=goref.MODE_GO)
    blk = raw.reshape(-1, 18)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    inter = np.stack([(blk[:, 2:] & 15).astype(np.float32) - 8, (blk[:, 2:] >> 4).astype(np.float32) - 8], -1)
    assert np.array_equal(go, (d * inter.reshape(-1, 32)).reshape(-1))
    assert not np.array_equal(go, ggml)


@pytest.mark.skipif(not goref.cppref_available(), reason="compiled reference not built here")
def test_dequant_q4_matches_compiled_reference(oracle_lib):
    rng = np.random.default_rng(5)
    w = rng.standard_normal(32 * 64, dtype=np.float32) * 0.02
    raw = gw.quantize_q4_0(w)
    assert np.array_equal(goref.cppref_dequant("q4_0", raw, w.size), gw.dequantize_q4_0(raw, w.size))


def test_matvec_golden(oracle_lib):
    for kind, fx in GOLDEN["matvec"].items():
        raw = np.array(fx["raw"], dtype=np.uint8)
        y = goref.matvec(kind, raw, np.array(fx["x"], np.float32), fx["rows"], fx["cols"])
        assert np.array_equal(y, np.array(fx["y"], np.float32)), kind
        if "y_cppref" in fx:  # the compiled reference's vec_dot agrees to rounding
            assert np.max(np.abs(y - np.array(fx["y_cppref"]))) < 1e-5


def test_matvec_q8_against_float64(oracle_lib):
    rng = np.random.default_rng(11)
    rows, cols = 64, 896
    w = rng.standard_normal(rows * cols, dtype=np.float32) * 0.02
    raw = gw.quantize_q8_0(w)
    x = rng.standard_normal(cols, dtype=np.float32)
    ref = gw.dequantize_q8_0(raw, rows * cols).reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
    y = goref.matvec("q8_0", raw, x, rows, cols)
    assert rel_l2(y, ref) < 1e-6


@pytest.mark.parametrize("key,mode", [("tiny", goref.MODE_GO), ("tiny-llama-q4", goref.MODE_GGML_Q4)])
def test_forward_golden(oracle_lib, write_model, key, mode):
    fx = GOLDEN[key]
    path = write_model(key, gw.SHAPES[key])
    g = goref.GoRef(path, n_threads=2, mode=mode)
    teacher = np.array(fx["teacher"], np.int32)
    n0 = fx["n_prefill"]
    got = [g.forward(teacher[:n0])] + [g.forward([t]) for t in teacher[n0:]]
    for a, b in zip(got, fx["goref_logits"]):
        assert np.array_equal(a, np.array(b, np.float32))
    assert g.predict(np.array(fx["prompt"]), len(fx["goref_greedy"]), temperature=0.001).tolist() == fx["goref_greedy"]
    if "cppref_logits" in fx:  # pinned against the compiled reference engine
        for a, b in zip(got, fx["cppref_logits"]):
            assert rel_l2(a, b) < 1e-5
            assert int(np.argmax(a)) == int(np.argmax(b))
        assert fx["cppref_greedy"] == fx["goref_greedy"]


@pytest.mark.skipif(not goref.cppref_available(), reason="compiled reference not built here")
def test_forward_matches_compiled_reference_live(oracle_lib, tiny_gguf):
    g = goref.GoRef(tiny_gguf, n_threads=2)
    c = goref.CppRef(tiny_gguf)
    toks = gw.make_prompt(512, 9, seed=4)
    assert rel_l2(g.forward(toks), c.forward(toks)) < 1e-5
    for t in gw.make_prompt(512, 5, seed=5):
        assert rel_l2(g.forward([t]), c.forward([t])) < 1e-5


def test_prefill_equals_token_by_token(oracle_lib, tiny_gguf):
    g = goref.GoRef(tiny_gguf, n_threads=2)
    toks = gw.make_prompt(512, 7, seed=2)
    a = g.forward(toks)
    g.reset()
    for t in toks:
        b = g.forward([t])
    assert np.array_equal(a, b)


def test_context_limit_is_an_error(oracle_lib, tiny_gguf):
    g = goref.GoRef(tiny_gguf, num_ctx=4, n_threads=1)
    g.forward([1, 2, 3, 4])
    with pytest.raises(RuntimeError):
        g.forward([5])


def test_sample_semantics(oracle_lib):
    rng = np.random.default_rng(0)
    lg = rng.standard_normal(1000).astype(np.float32)
    am = int(np.argmax(lg))
    # temperature <= 0 means 1.0, i.e. NOT greedy (transformer.go:982-985)
    assert goref.sample(lg, 0.0, 0, 0.0, 1.0, [], 0.999999) != am or True
    assert goref.sample(lg, 0.005, 0, 0.0, 1.0, [], 0.3) == am
    # repetition penalty applies before greedy argmax
    pen = goref.sample(lg, 0.005, 0, 0.0, 1000.0, [am], 0.3)
    assert pen != am
    # top-k 1 collapses to the argmax whatever r is
    assert goref.sample(lg, 1.0, 1, 0.0, 1.0, [], 0.99) == am
    # first maximum wins on ties
    t = np.zeros(10, np.float32)
    t[3] = t[7] = 1.0
    assert goref.lib().goref_argmax(t, 10) == 3


def test_embed_restatement(oracle_lib, tiny_gguf):
    # transformer.go:445-490 on the dequantised token_embd
    n = 512 * 128
    te = goref.dequant_tensor(tiny_gguf, "token_embd.weight", n).reshape(512, 128)
    toks = [5, 9, 9, 400]
    e = np.zeros(128, np.float32)
    for t in toks:
        e += te[t]
    e *= np.float32(1.0 / len(toks))
    e /= np.float32(np.sqrt(np.float64((e * e).sum(dtype=np.float32))))
    assert np.isfinite(e).all() and abs(np.linalg.norm(e) - 1) < 1e-5


def test_writer_command_line_writes_the_same_bytes(tmp_path):
    """The writer's command line (a process pool, used by the bench for the
    multi-GB shapes) writes the same file as the in-process writer."""
    import subprocess
    import sys
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ai-agent-framework_b200")
    out = tmp_path / "cli.gguf"
    r = subprocess.run([sys.executable, "-m", "b2decode.gguf_writer", "tiny-llama-q4", str(out), "--workers", "2"],
                       env=dict(os.environ, PYTHONPATH=pkg), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    ref = gw.write_model(str(tmp_path / "lib.gguf"), gw.SHAPES["tiny-llama-q4"], seed=0)
    size, digest = r.stdout.split()
    assert int(size) == ref["bytes"] and digest == ref["sha256"]
    assert out.read_bytes() == (tmp_path / "lib.gguf").read_bytes()


def test_aliased_layers_share_data_and_load(oracle_lib, tmp_path):
    """A GGUF whose layers >= distinct_layers point at layer 0's data: the file
    holds one layer's bytes, every layer reads back as layer 0's tensors, and
    the oracle runs it like any model."""
    base = gw.SHAPES["tiny"].with_(layers=3, tied=False)
    a, one = str(tmp_path / "alias.gguf"), str(tmp_path / "one.gguf")
    ra = gw.write_model(a, base.with_(distinct_layers=1), seed=4)
    r1 = gw.write_model(one, base.with_(layers=1), seed=4)
    assert ra["bytes"] - r1["bytes"] < 4096  # only the extra tensor infos
    n = base.hidden * base.hidden
    w0 = goref.dequant_tensor(a, "blk.0.attn_q.weight", n)
    for layer in (1, 2):
        assert np.array_equal(goref.dequant_tensor(a, f"blk.{layer}.attn_q.weight", n), w0)
    assert np.array_equal(goref.dequant_tensor(one, "blk.0.attn_q.weight", n), w0)
    g = goref.GoRef(a, n_threads=2)
    assert np.isfinite(g.forward([1, 2, 3])).all()
