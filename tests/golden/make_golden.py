"""Regenerates tests/golden/*.json.

Run in the development container, where the reference sources exist so the
compiled C++ sibling engine (oracle/_ref/libcppref.so) can be built:

    python tests/golden/make_golden.py

Each fixture records the synthetic model's sha256 (pinning the writer), the
goref oracle's outputs and, where available, the compiled reference engine's
outputs on the same inputs.  Tests compare the oracle against these files and
the GPU engine against the oracle.
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "ai-agent-framework_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import goref  # noqa: E402
from b2decode import gguf_writer as gw  # noqa: E402


def r32(a):
    return [float(np.float32(v)) for v in np.asarray(a, dtype=np.float32).reshape(-1)]


def model_fixture(name, shape, mode, n_prompt=12, n_greedy=24):
    tmp = tempfile.mkdtemp()
    path = os.path.join(tmp, name + ".gguf")
    info = gw.write_model(path, shape, seed=0)
    g = goref.GoRef(path, n_threads=4, mode=mode)
    prompt = gw.make_prompt(shape.vocab, n_prompt, seed=0)
    teacher = np.concatenate([[g.cfg["bos_id"]], prompt, gw.make_prompt(shape.vocab, 6, seed=1)]).astype(np.int32)
    # teacher-forced: prefill the first n_prompt+1 ids, then one id at a time
    g.reset()
    steps = [g.forward(teacher[: n_prompt + 1])]
    for t in teacher[n_prompt + 1:]:
        steps.append(g.forward([t]))
    greedy = g.predict(prompt, n_greedy, temperature=0.001).tolist()
    out = {
        "shape": shape.__dict__, "seed": 0, "sha256": info["sha256"], "bytes": info["bytes"],
        "mode": mode, "prompt": prompt.tolist(), "teacher": teacher.tolist(), "n_prefill": n_prompt + 1,
        "goref_logits": [r32(s) for s in steps], "goref_greedy": greedy,
    }
    if goref.cppref_available() and mode == goref.MODE_GO:
        c = goref.CppRef(path)
        cs = [c.forward(teacher[: n_prompt + 1])]
        for t in teacher[n_prompt + 1:]:
            cs.append(c.forward([t]))
        out["cppref_logits"] = [r32(s) for s in cs]
        c.reset()
        ids, lg = [], c.forward(np.concatenate([[g.cfg["bos_id"]], prompt]))
        for _ in range(n_greedy):
            t = int(np.argmax(lg))
            ids.append(t)
            lg = c.forward([t])
        out["cppref_greedy"] = ids
    return out


def matvec_fixture():
    rng = np.random.default_rng(7)
    out = {}
    for kind, rows, cols in (("q8_0", 48, 256), ("q4_0", 40, 320)):
        w = (rng.standard_normal(rows * cols, dtype=np.float32) * 0.02)
        x = rng.standard_normal(cols, dtype=np.float32)
        raw = gw.quantize(w, gw.TYPE_NAMES[kind])
        y = goref.matvec(kind, raw, x, rows, cols)
        out[kind] = {"rows": rows, "cols": cols, "w_seed": 7, "raw": raw.tolist(), "x": r32(x), "y": r32(y)}
        if goref.cppref_available():
            L = goref.cpplib()
            rb = raw.size // rows
            fn = L.cppref_vec_dot_q8_0 if kind == "q8_0" else L.cppref_vec_dot_q4_0
            out[kind]["y_cppref"] = [float(fn(np.ascontiguousarray(raw[r * rb:(r + 1) * rb]), x, cols))
                                     for r in range(rows)]
    return out


if __name__ == "__main__":
    goref.build()
    fx = {
        "tiny": model_fixture("tiny", gw.SHAPES["tiny"], goref.MODE_GO),
        "tiny-llama-q4": model_fixture("tiny-llama-q4", gw.SHAPES["tiny-llama-q4"], goref.MODE_GGML_Q4),
        "matvec": matvec_fixture(),
    }
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(fx, f)
    print("wrote", os.path.join(HERE, "golden.json"), os.path.getsize(os.path.join(HERE, "golden.json")), "bytes")
