"""Batched greedy decode (b2_batch_*) against the oracle.

Three sequences with prompts of different lengths share the batch; every
step's logits of every slot are compared with the oracle run on that
sequence alone with the same token history (teacher-forced on the batch's
own ids): within the logits bar of the single-sequence path (1e-2 relative
L2 per step) and the same argmax on at least 99% of the steps.
"""
import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


SHAPES = {
    # head dim 64, QKV bias, tied embeddings
    "qwen2-hd64-q8": gw.ModelShape("qwen2", 256, 2, 4, 2, 512, 512, 256, 1e-6, 1e6, True, True, "q8_0", 1, 2),
    # head dim 128, GQA group 4, untied Q4_0 lm_head
    "llama-hd128-q4": gw.ModelShape("llama", 512, 2, 4, 1, 1024, 384, 256, 1e-5, 5e5, False, False, "q4_0", 1, 2),
}


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("key", list(SHAPES))
def test_batch_decode_matches_oracle_per_sequence(built_lib, oracle_lib, write_model, key, graph):
    """graph: steps after the first replay a captured CUDA graph."""
    shape = SHAPES[key]
    path = write_model(key, shape)
    m = b2decode.Model(path, num_ctx=128)
    mode = goref.MODE_GGML_Q4 if shape.wtype == "q4_0" else goref.MODE_GO
    g = goref.GoRef(path, num_ctx=128, n_threads=0, mode=mode)
    prompts = [np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, n, seed=10 + n)]).astype(np.int32)
               for n in (5, 70, 1)]
    bt = b2decode.Batch(m, len(prompts))
    if graph:
        bt.use_graph(True)
    hist = [list(p) for p in prompts]
    nxt = []
    for slot, p in enumerate(prompts):
        first = bt.prefill(slot, p)
        g.reset()
        want = g.forward(p)
        assert first == int(np.argmax(want)), slot
        nxt.append(first)
    agree, errs = [], []
    for _ in range(8):
        ids = bt.step(nxt)
        lg = bt.logits()
        for slot in range(len(prompts)):
            hist[slot].append(nxt[slot])
            g.reset()
            want = g.forward(np.array(hist[slot], np.int32))
            errs.append(rel_l2(lg[slot], want))
            agree.append(int(ids[slot]) == int(np.argmax(want)))
        nxt = [int(i) for i in ids]
    assert max(errs) < LOGIT_TOL, errs
    assert np.mean(agree) >= 0.99, agree
    bt.close()
    m.close()


def test_batch_rejects_what_it_cannot_run(built_lib, write_model):
    shape = gw.SHAPES["tiny"]  # head dim 32: not a batched-attention geometry
    m = b2decode.Model(write_model("tiny-batch", shape), num_ctx=64)
    with pytest.raises(b2decode.B2Error) as e:
        b2decode.Batch(m, 2)
    assert e.value.code == -3
    m.close()
    m = b2decode.Model(write_model("hd64-batch", SHAPES["qwen2-hd64-q8"]), num_ctx=16)
    for bad in (0, 17):
        with pytest.raises(b2decode.B2Error):
            b2decode.Batch(m, bad)
    bt = b2decode.Batch(m, 2)
    with pytest.raises(b2decode.B2Error) as e:
        bt.prefill(2, [1, 2, 3])
    assert e.value.code == -8
    with pytest.raises(b2decode.B2Error) as e:
        bt.prefill(0, list(range(1, 17)))  # no room for a generated token
    assert e.value.code == -9
    bt.close()
    m.close()


def test_batch_prefill_long_prompt_chunks(built_lib, oracle_lib, write_model):
    """A 300-token prompt runs in two chunks of 150 tokens on the
    tensor-core GEMM, the second attending over the cache the first
    wrote: the argmax after the prompt, its logits (row 0) and four steps
    after it against the oracle."""
    shape = SHAPES["llama-hd128-q4"].with_(context=512)
    path = write_model("llama-hd128-q4-ctx512", shape)
    m = b2decode.Model(path, num_ctx=320)
    g = goref.GoRef(path, num_ctx=320, n_threads=0, mode=goref.MODE_GGML_Q4)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 299, seed=21)]).astype(np.int32)
    bt = b2decode.Batch(m, 1)
    first = bt.prefill(0, prompt)
    want = g.forward(prompt)
    assert rel_l2(bt.logits()[0], want) < LOGIT_TOL
    assert first == int(np.argmax(want))
    nxt, errs = [first], []
    for _ in range(4):
        ids = bt.step(nxt)
        want = g.forward(nxt)
        errs.append(rel_l2(bt.logits()[0], want))
        assert int(ids[0]) == int(np.argmax(want))
        nxt = [int(ids[0])]
    assert max(errs) < LOGIT_TOL, errs
    bt.close()
    m.close()
