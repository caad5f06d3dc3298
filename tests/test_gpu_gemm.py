"""b2_model_gemm, the tcgen05 tensor-core GEMM over the resident tiled
weights (the prefill and batched-step product), against the dequantised
tensor (bit-exact with the oracle) times X in float64.

Two bars per output vector:
* against the exact product: 3e-3 relative L2 (the operands are rounded to
  fp16 once: d * q of each weight, and each activation after a power-of-two
  scale per token, 2^-12 relative at most; sums in fp32);
* against the same product with the operands rounded to fp16 exactly as the
  kernel rounds them: 2e-5 (what is left is fp32 summation order), which
  checks the data path itself: the TMA boxes, the 128-byte swizzle, the
  descriptors, the split over K.
"""
import numpy as np
import pytest

import b2decode
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu

TOL_EXACT = 3e-3
TOL_ROUNDED = 2e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def fp16_scaled(x):
    """Each row times 2^e (its largest magnitude into [2^14, 2^15)), rounded
    to fp16, then scaled back: the activations the kernel multiplies."""
    out = np.empty_like(x, dtype=np.float64)
    for t in range(x.shape[0]):
        mx = float(np.abs(x[t]).max())
        e = 0
        if mx > 0:
            e = 15 - int(np.frexp(mx)[1])
        out[t] = (x[t].astype(np.float64) * 2.0 ** e).astype(np.float16).astype(np.float64) * 2.0 ** -e
    return out


MODEL_SHAPES = {
    "tiny-q8": gw.SHAPES["tiny"],
    "tiny-llama-q4": gw.SHAPES["tiny-llama-q4"],
    "wide-q4": gw.ModelShape("llama", 1024, 1, 8, 2, 2816, 1000, 256, 1e-5, 5e5, False, False, "q4_0", 1, 2),
    "wide-q8": gw.ModelShape("qwen2", 1024, 1, 8, 2, 2816, 1000, 256, 1e-6, 1e6, True, False, "q8_0", 1, 2),
}


@pytest.mark.parametrize("key", list(MODEL_SHAPES))
def test_gemm_over_resident_tiled_weights(built_lib, torch_cuda, write_model, key):
    torch = torch_cuda
    shape = MODEL_SHAPES[key]
    m = b2decode.Model(write_model(key, shape), num_ctx=64)
    H, qd, kvd, ff, V = shape.hidden, shape.hidden, shape.kv_dim, shape.ffn, shape.vocab
    dims = {"blk.0.attn_q.weight": (qd, H), "blk.0.attn_k.weight": (kvd, H), "blk.0.attn_v.weight": (kvd, H),
            "blk.0.attn_output.weight": (H, qd), "blk.0.ffn_down.weight": (H, ff), "token_embd.weight": (V, H)}
    if not shape.tied:
        dims["output.weight"] = (V, H)
    dims["blk.0.ffn_gate.weight"] = (ff, H)  # the two halves of the interleaved resident matrix
    dims["blk.0.ffn_up.weight"] = (ff, H)
    rng = np.random.default_rng(11)
    for name, (rows, cols) in dims.items():
        w = m.dequant(name, rows * cols).reshape(rows, cols)
        w64 = w.astype(np.float64)
        w16 = w.astype(np.float16).astype(np.float64)
        for ntok in (1, 7, 16, 40, 100, 130, 300):
            x = rng.standard_normal((ntok, cols), dtype=np.float32)
            x[0, :32] *= 1e-3
            dx = torch.from_numpy(x).cuda()
            dy = torch.full((ntok, rows), float("nan"), device="cuda")
            m.gemm(name, dx.data_ptr(), dy.data_ptr(), ntok)
            torch.cuda.synchronize()
            got = dy.cpu().numpy()
            assert np.isfinite(got).all(), (name, ntok)
            exact = x.astype(np.float64) @ w64.T
            rounded = fp16_scaled(x) @ w16.T
            for t in {0, ntok // 2, ntok - 1}:
                assert rel_l2(got[t], exact[t]) < TOL_EXACT, (name, ntok, t, rel_l2(got[t], exact[t]))
                assert rel_l2(got[t], rounded[t]) < TOL_ROUNDED, (name, ntok, t, rel_l2(got[t], rounded[t]))
    m.close()


def test_gemm_large_k_split_and_deterministic(built_lib, torch_cuda, write_model):
    """A long K (FFN 2816 -> 44 stages) with few row tiles is split over K
    and summed in split order: equal inputs give equal bits, and a zero
    token row gives zeros."""
    torch = torch_cuda
    shape = MODEL_SHAPES["wide-q4"]
    m = b2decode.Model(write_model("wide-q4", shape), num_ctx=64)
    rows, cols = shape.hidden, shape.ffn
    name = "blk.0.ffn_down.weight"
    w = m.dequant(name, rows * cols).reshape(rows, cols).astype(np.float16).astype(np.float64)
    x = np.random.default_rng(5).standard_normal((9, cols), dtype=np.float32)
    x[4] = 0.0
    dx = torch.from_numpy(x).cuda()
    outs = []
    for _ in range(2):
        dy = torch.full((9, rows), float("nan"), device="cuda")
        m.gemm(name, dx.data_ptr(), dy.data_ptr(), 9)
        torch.cuda.synchronize()
        outs.append(dy.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert np.all(outs[0][4] == 0.0)
    want = fp16_scaled(x) @ w.T
    for t in (0, 3, 8):
        assert rel_l2(outs[0][t], want[t]) < TOL_ROUNDED
    m.close()


@pytest.mark.parametrize("key", ["qwen2-hd64-q8", "llama-hd128-q4"])
def test_model_prefill_on_tensor_cores(built_lib, oracle_lib, write_model, key):
    """b2_forward with a prompt of 16+ tokens runs the prefill on the GEMM
    path into the model's own cache (one chunk of 200 tokens); the same prompt fed one token per decode-kernel launch, and the
    oracle, give the same logits to 1e-2 relative L2 and the same argmax;
    decode steps after either prefill agree too."""
    import goref
    shapes = {
        "qwen2-hd64-q8": gw.ModelShape("qwen2", 256, 2, 4, 2, 512, 512, 512, 1e-6, 1e6, True, True, "q8_0", 1, 2),
        "llama-hd128-q4": gw.ModelShape("llama", 512, 2, 4, 1, 1024, 384, 512, 1e-5, 5e5, False, False, "q4_0", 1, 2),
    }
    shape = shapes[key]
    path = write_model(key + "-prefill", shape)
    gemm = b2decode.Model(path, num_ctx=256)
    step = b2decode.Model(path, num_ctx=256)
    mode = goref.MODE_GGML_Q4 if shape.wtype == "q4_0" else goref.MODE_GO
    g = goref.GoRef(path, num_ctx=256, n_threads=0, mode=mode)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 199, seed=12)]).astype(np.int32)
    a = gemm.forward(prompt)
    for t in prompt[:-1]:
        step.forward([int(t)])
    b = step.forward([int(prompt[-1])])
    c = g.forward(prompt)
    assert gemm.cache_len == step.cache_len == 200
    assert rel_l2(a, c) < 1e-2 and rel_l2(b, c) < 1e-2, (rel_l2(a, c), rel_l2(b, c))
    assert int(np.argmax(a)) == int(np.argmax(c)) == int(np.argmax(b))
    t = int(np.argmax(c))
    for _ in range(4):
        x, y, z = gemm.forward([t]), step.forward([t]), g.forward([t])
        assert rel_l2(x, z) < 1e-2 and rel_l2(y, z) < 1e-2
        t = int(np.argmax(z))
    gemm.close()
    step.close()


def test_model_prefill_in_chunks_continues_the_cache(built_lib, oracle_lib, write_model):
    """b2_forward with a 300-token prompt: two chunks of 150 tokens on the
    GEMM path, the second attending over the cache the first wrote; then a
    second call of 40 tokens continues the same cache from position 300 (one
    more chunk), and a decode step follows.  Logits and argmax against the
    oracle after each call."""
    import goref
    shape = gw.ModelShape("llama", 512, 2, 4, 1, 1024, 384, 512, 1e-5, 5e5, False, False, "q4_0", 1, 2)
    path = write_model("llama-hd128-q4-chunks", shape)
    m = b2decode.Model(path, num_ctx=400)
    g = goref.GoRef(path, num_ctx=400, n_threads=0, mode=goref.MODE_GGML_Q4)
    # (seeds whose top-1 logit leads the next by over 0.15 rms at every check)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 299, seed=33)]).astype(np.int32)
    more = gw.make_prompt(shape.vocab, 40, seed=133).astype(np.int32)
    for toks, pos in ((prompt, 300), (more, 340)):
        a, c = m.forward(toks), g.forward(toks)
        assert m.cache_len == pos
        assert rel_l2(a, c) < 1e-2, (pos, rel_l2(a, c))
        assert int(np.argmax(a)) == int(np.argmax(c)), pos
    t = int(np.argmax(c))
    a, c = m.forward([t]), g.forward([t])
    assert rel_l2(a, c) < 1e-2 and int(np.argmax(a)) == int(np.argmax(c))
    m.close()
