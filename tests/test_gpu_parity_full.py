"""Parity at the benchmarked sizes, through the C ABI against the oracle.

* Config 0 exactly as the decode benchmark runs it: the Qwen2.5-0.5B shape
  (Q8_0, all 24 layers, vocab 151936), BOS + 128 prompt ids from seed 0,
  prefill, then 128 greedy decode steps.  Every step's logits are compared
  with the oracle teacher-forced on the engine's own greedy ids (relative L2
  per step within 1e-2, top-1 agreement >= 99%), and the device-resident
  greedy loop (b2_decode_greedy) must emit exactly the ids of the per-step
  path.
* Config 2 at its real matrix shapes: the Llama-3-8B widths (hidden 4096, 32 /
  8 heads of 128, FFN 14336, vocab 128256, untied, Q4_0) cut to 4 layers,
  against the oracle's ggml-order Q4_0 mode.

Reference loops: transformer.go:325-382 (Predict), 519-739 (forward).
"""
import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2   # relative L2 per step
TOP1 = 0.99        # teacher-forced top-1 agreement


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def run_teacher_forced(m, g, prompt, steps):
    """Prefill both engines with the prompt, then feed the engine's greedy id
    to both for `steps` steps.  Returns (errors, top-1 agreements, ids fed,
    the engine's argmax after the last step)."""
    a, b = m.forward(prompt), g.forward(prompt)
    errs, agree, ids = [rel_l2(a, b)], [int(np.argmax(a)) == int(np.argmax(b))], []
    t = int(np.argmax(a))
    for _ in range(steps):
        ids.append(t)
        a, b = m.forward([t]), g.forward([t])
        errs.append(rel_l2(a, b))
        agree.append(int(np.argmax(a)) == int(np.argmax(b)))
        t = int(np.argmax(a))
    return errs, agree, ids, t


def test_qwen05b_full_length(built_lib, oracle_lib, write_model):
    shape = gw.SHAPES["qwen2.5-0.5b"]
    path = write_model("qwen05b", shape)
    m = b2decode.Model(path, num_ctx=512)
    g = goref.GoRef(path, num_ctx=512, n_threads=0)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 128, seed=0)]).astype(np.int32)
    errs, agree, ids, last = run_teacher_forced(m, g, prompt, 128)
    assert len(errs) == 129
    assert max(errs) < LOGIT_TOL, (max(errs), int(np.argmax(errs)))
    assert np.mean(agree) >= TOP1, np.mean(agree)
    # the device-resident loop from the same prefix emits the same ids
    m.reset()
    first = m.forward_argmax(prompt)
    assert first == ids[0]
    got = m.decode_greedy(first, 128)
    assert got.tolist() == ids[1:] + [last]
    m.close()


def test_llama8b_width_q4_parity(built_lib, oracle_lib, write_model):
    shape = gw.SHAPES["llama3-8b-4l"]
    path = write_model("llama3-8b-4l", shape)
    m = b2decode.Model(path, num_ctx=256)
    g = goref.GoRef(path, num_ctx=256, n_threads=0, mode=goref.MODE_GGML_Q4)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 40, seed=2)]).astype(np.int32)
    errs, agree, ids, last = run_teacher_forced(m, g, prompt, 12)
    assert max(errs) < LOGIT_TOL, errs
    assert np.mean(agree) >= TOP1, agree
    m.reset()
    first = m.forward_argmax(prompt)
    assert first == ids[0]
    assert m.decode_greedy(first, 12).tolist() == ids[1:] + [last]
    m.close()
