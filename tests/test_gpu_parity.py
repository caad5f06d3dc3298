"""Parity of the CUDA path (called through the C ABI) with the oracle.

Bars (from the reference contract): dequantised weights and greedy token ids
bit-exact; teacher-forced logits within 1e-2 relative L2 per step; greedy
top-1 agreement >= 99%.  Kernel-level entry points are checked against the
oracle's restatement of the same Go loops.
"""
import os

import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2      # relative L2 per step
TIGHT_TOL = 1e-4      # what fp32 math actually achieves with an fp32 KV cache


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def teacher_forced(engine_fwd, oracle_fwd, tokens, n_prefill):
    out = []
    a = engine_fwd(tokens[:n_prefill])
    b = oracle_fwd(tokens[:n_prefill])
    out.append((a, b))
    for t in tokens[n_prefill:]:
        out.append((engine_fwd([t]), oracle_fwd([t])))
    return out


@pytest.mark.parametrize("kv_fp32", [False, True])
def test_tiny_teacher_forced_logits(built_lib, oracle_lib, tiny_gguf, kv_fp32):
    m = b2decode.Model(tiny_gguf, kv_fp32=kv_fp32)
    g = goref.GoRef(tiny_gguf, n_threads=4)
    toks = np.concatenate([[1], gw.make_prompt(512, 20, seed=3), gw.make_prompt(512, 30, seed=4)]).astype(np.int32)
    pairs = teacher_forced(m.forward, g.forward, toks, 21)
    errs = [rel_l2(a, b) for a, b in pairs]
    agree = np.mean([int(np.argmax(a)) == int(np.argmax(b)) for a, b in pairs])
    assert max(errs) < (TIGHT_TOL if kv_fp32 else LOGIT_TOL), errs
    assert agree >= 0.99
    assert m.cache_len == g.cache_len == len(toks)


def test_tiny_greedy_ids_exact(built_lib, oracle_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf)
    g = goref.GoRef(tiny_gguf, n_threads=4)
    for seed in range(3):
        prompt = gw.make_prompt(512, 10 + seed, seed=seed)
        want = g.predict(prompt, 40, temperature=0.001)
        got, tim = m.predict(prompt, b2decode.sample_opts(temperature=0.001, num_predict=40))
        assert got.tolist() == want.tolist()
        assert tim["prompt_tokens"] == len(prompt) + 1


def test_device_loop_equals_stepwise(built_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf)
    prompt = np.concatenate([[1], gw.make_prompt(512, 9, seed=9)])
    first = m.forward_argmax(prompt)
    ids = m.decode_greedy(first, 25)
    m.reset()
    t = m.forward_argmax(prompt)
    step = []
    for _ in range(25):
        t2 = m.forward_argmax([t])
        step.append(t2)
        t = t2
    assert ids.tolist() == step


def test_decode_greedy_eos_stops(built_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf)
    prompt = np.concatenate([[1], gw.make_prompt(512, 9, seed=9)])
    first = m.forward_argmax(prompt)
    ids = m.decode_greedy(first, 12)
    m.reset()
    m.forward_argmax(prompt)
    eos = int(ids[4])
    k = ids.tolist().index(eos)
    got = m.decode_greedy(first, 12, eos=eos)
    assert got.tolist() == ids[:k].tolist()
    assert m.cache_len == len(prompt) + k + 1


def test_stream_matches_predict(built_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf)
    prompt = gw.make_prompt(512, 8, seed=1)
    opts = b2decode.sample_opts(temperature=0.001, num_predict=16)
    want, _ = m.predict(prompt, opts)
    got = list(m.stream(prompt, opts))
    assert got == want.tolist()


def test_sampled_predict_with_fixed_uniforms(built_lib, oracle_lib, tiny_gguf):
    # The host sampler (b2_sample_logits) over the engine's logits picks what
    # sample() picks with the same uniforms (the device sampler has its own
    # tests).
    m = b2decode.Model(tiny_gguf, kv_fp32=True)
    g = goref.GoRef(tiny_gguf, n_threads=4)
    toks = np.concatenate([[1], gw.make_prompt(512, 6, seed=7)])
    a = m.forward(toks)
    b = g.forward(toks)
    for temp, k, p, rp in ((0.8, 40, 0.9, 1.3), (1.0, 0, 0.0, 1.0), (0.001, 0, 0.0, 1.3)):
        for r in (0.05, 0.5, 0.95):
            opts = b2decode.sample_opts(temp, k, p, rp)
            assert b2decode.sample_logits(a, opts, [3, 5], r) == goref.sample(b, temp, k, p, rp, [3, 5], r)


def test_dequant_bit_exact(built_lib, oracle_lib, tiny_gguf, tiny_q4_gguf):
    for path, mode in ((tiny_gguf, goref.MODE_GO), (tiny_q4_gguf, goref.MODE_GGML_Q4)):
        m = b2decode.Model(path)
        for name in ("token_embd.weight", "blk.0.attn_q.weight", "blk.1.attn_v.weight", "blk.1.ffn_down.weight",
                     "blk.0.ffn_up.weight", "output_norm.weight"):
            n = 1 << 20
            want = goref.dequant_tensor(path, name, n, mode=mode)
            got = m.dequant(name, n)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


def test_q4_model_teacher_forced(built_lib, oracle_lib, tiny_q4_gguf):
    m = b2decode.Model(tiny_q4_gguf, kv_fp32=True)
    g = goref.GoRef(tiny_q4_gguf, n_threads=4, mode=goref.MODE_GGML_Q4)
    toks = np.concatenate([[1], gw.make_prompt(384, 12, seed=5), gw.make_prompt(384, 20, seed=6)]).astype(np.int32)
    pairs = teacher_forced(m.forward, g.forward, toks, 13)
    assert max(rel_l2(a, b) for a, b in pairs) < TIGHT_TOL
    want = g.predict(gw.make_prompt(384, 12, seed=5), 24, temperature=0.001)
    got, _ = m.predict(gw.make_prompt(384, 12, seed=5), b2decode.sample_opts(temperature=0.001, num_predict=24))
    assert got.tolist() == want.tolist()


def test_embed(built_lib, oracle_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf)
    te = goref.dequant_tensor(tiny_gguf, "token_embd.weight", 512 * 128).reshape(512, 128)
    for toks in ([5], [5, 9, 9, 400], list(range(0, 500, 7)), [3, 100000, 4]):
        e = np.zeros(128, np.float32)
        for t in toks:
            if 0 <= t < 512:
                e += te[t]
        e *= np.float32(1.0 / len(toks))
        e /= np.float32(np.sqrt(np.float64((e * e).sum(dtype=np.float32))))
        assert np.allclose(m.embed(toks), e, rtol=1e-5, atol=1e-6)
    assert not m.embed([]).any()


def test_load_stats(built_lib, tiny_gguf):
    # the weights travel through the mapped file and the pinned stages: every
    # matrix byte of the file once, and the phases add up
    import gguf
    quant = sum(int(t.n_bytes) for t in gguf.GGUFReader(tiny_gguf).tensors
                if t.tensor_type in (gguf.GGMLQuantizationType.Q8_0, gguf.GGMLQuantizationType.Q4_0))
    m = b2decode.Model(tiny_gguf)
    s = m.load_stats()
    assert s["mapped"] == 1 and s["host_threads"] >= 1
    assert s["bytes_uploaded"] == quant
    assert 0 < s["parse_ns"] < s["total_ns"] and 0 < s["upload_ns"] < s["total_ns"]
    assert 0 <= s["host_copy_ns"] <= s["upload_ns"]
    m.close()


def test_context_overflow_and_reset(built_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf, num_ctx=16)
    m.forward(list(range(1, 17)))
    with pytest.raises(b2decode.B2Error) as e:
        m.forward([3])
    assert e.value.code == -9
    m.reset()
    assert m.cache_len == 0
    m.forward([1, 2, 3])


def test_out_of_range_token_embeds_zero(built_lib, oracle_lib, tiny_gguf):
    m = b2decode.Model(tiny_gguf, kv_fp32=True)
    g = goref.GoRef(tiny_gguf, n_threads=2)
    toks = [1, 700, -5, 4]
    assert rel_l2(m.forward(toks), g.forward(toks)) < TIGHT_TOL


def test_bounded_wait_reports_timeout(built_lib, tiny_gguf):
    # A wait that nothing will satisfy runs out (about 2 s), the kernel returns
    # and the host reads B2_ERR_TIMEOUT; the context stays usable.
    m = b2decode.Model(tiny_gguf)
    m.debug_wait_skew(1000)
    with pytest.raises(b2decode.B2Error) as e:
        m.forward([1, 2])
    assert e.value.code == -7
    m.reset()
    a = m.forward([1, 2, 3])
    m.reset()
    assert np.array_equal(a, m.forward([1, 2, 3]))


@pytest.mark.parametrize("kind", ["q8_0", "q4_0"])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096), (130, 96)])
def test_matvec_config1_shapes(built_lib, oracle_lib, torch_cuda, kind, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows ^ cols)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    raw = gw.quantize(w, gw.TYPE_NAMES[kind])
    x = rng.standard_normal(cols, dtype=np.float32)
    want = goref.matvec(kind, raw, x, rows, cols)
    dw = torch.from_numpy(raw).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((rows,), float("nan"), device="cuda")
    b2decode.matvec(8 if kind == "q8_0" else 2, dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    assert np.isfinite(got).all()
    # same products, different summation order: fp32 rounding only
    assert rel_l2(got, want) < 1e-5
    assert np.max(np.abs(got - want)) <= 1e-4 * np.max(np.abs(want)) + 1e-6


@pytest.mark.parametrize("kind,rows,cols", [("q8_0", 300, 32768), ("q4_0", 300, 32768)])
def test_matvec_small_ring(built_lib, oracle_lib, torch_cuda, kind, rows, cols):
    """Rows so wide that the shared-memory ring has fewer slots (2 for Q8_0) than
    the producer has lanes and the kernel has consumer warps: checks that the
    producer never puts two chunks of one slot in a batch and that consumers
    wait for a chunk to be issued before waiting on its slot."""
    torch = torch_cuda
    rng = np.random.default_rng(rows + cols)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    raw = gw.quantize(w, gw.TYPE_NAMES[kind])
    x = rng.standard_normal(cols, dtype=np.float32)
    want = goref.matvec(kind, raw, x, rows, cols)
    dw = torch.from_numpy(raw).cuda()
    dx = torch.from_numpy(x).cuda()
    for _ in range(2):
        dy = torch.full((rows,), float("nan"), device="cuda")
        b2decode.matvec(8 if kind == "q8_0" else 2, dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols)
        torch.cuda.synchronize()
        got = dy.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, want) < 1e-5


@pytest.mark.parametrize("batch,ctx", [(1, 1), (1, 7), (2, 65), (1, 4096), (8, 4096), (1, 16384), (1, 32768)])
def test_attention_config3(built_lib, oracle_lib, torch_cuda, batch, ctx):
    torch = torch_cuda
    nh, nkv, hd = 32, 8, 128
    rng = np.random.default_rng(ctx + batch)
    q = rng.standard_normal((batch, nh * hd), dtype=np.float32)
    k = rng.standard_normal((batch, ctx, nkv * hd), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((batch, ctx, nkv * hd), dtype=np.float32).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty((batch, nh * hd), device="cuda")
    b2decode.attention_decode(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), batch, nh, nkv, hd, ctx)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    n_check = batch if ctx <= 4096 else 1
    for b in range(n_check):
        want = goref.attention(q[b], k[b].astype(np.float32), v[b].astype(np.float32), nh, nkv, hd, ctx)
        assert rel_l2(got[b], want) < 1e-4, (b, rel_l2(got[b], want))


def test_qwen05b_shape_parity(built_lib, oracle_lib, write_model):
    """The measured Qwen2.5-0.5B shape (all 24 layers, vocab 151936): teacher-
    forced logits and greedy ids against the oracle."""
    shape = gw.SHAPES["qwen2.5-0.5b"]
    path = write_model("qwen05b", shape)
    m = b2decode.Model(path, num_ctx=512)
    g = goref.GoRef(path, num_ctx=512, n_threads=0)
    prompt = gw.make_prompt(shape.vocab, 24, seed=0)
    toks = np.concatenate([[shape.bos_id], prompt, gw.make_prompt(shape.vocab, 8, seed=1)]).astype(np.int32)
    pairs = teacher_forced(m.forward, g.forward, toks, 25)
    errs = [rel_l2(a, b) for a, b in pairs]
    assert max(errs) < LOGIT_TOL, errs
    assert np.mean([int(np.argmax(a)) == int(np.argmax(b)) for a, b in pairs]) >= 0.99
    want = g.predict(prompt, 12, temperature=0.001)
    got, _ = m.predict(prompt, b2decode.sample_opts(temperature=0.001, num_predict=12))
    assert got.tolist() == want.tolist()


@pytest.mark.parametrize("arch,wtype,bias", [("llama", "q4_0", False), ("qwen2", "q8_0", True)])
def test_wide_heads_distributed_qa(built_lib, oracle_lib, write_model, arch, wtype, bias):
    """Head dim 128 over hidden 2048: one head's q rows exceed the fused QA
    phase's share, so the q, k, v rows are spread over all CTAs and each q CTA
    reads its head's q back; context past one attention tile (64 positions),
    so several splits.  Teacher-forced logits and greedy ids vs the oracle."""
    shape = gw.ModelShape(arch, 2048, 2, 16, 4, 1024, 1024, 512, 1e-5, 5e5, bias, not bias, wtype, 1, 2)
    path = write_model(f"wide-{arch}-{wtype}", shape)
    m = b2decode.Model(path, num_ctx=256)
    mode = goref.MODE_GGML_Q4 if wtype == "q4_0" else goref.MODE_GO
    g = goref.GoRef(path, num_ctx=256, n_threads=0, mode=mode)
    prompt = gw.make_prompt(shape.vocab, 70, seed=5)
    toks = np.concatenate([[shape.bos_id], prompt, gw.make_prompt(shape.vocab, 12, seed=6)]).astype(np.int32)
    pairs = teacher_forced(m.forward, g.forward, toks, 71)
    errs = [rel_l2(a, b) for a, b in pairs]
    assert max(errs) < LOGIT_TOL, errs
    assert np.mean([int(np.argmax(a)) == int(np.argmax(b)) for a, b in pairs]) >= 0.99
    want = g.predict(prompt, 8, temperature=0.001)
    got, _ = m.predict(prompt, b2decode.sample_opts(temperature=0.001, num_predict=8))
    assert got.tolist() == want.tolist()


def test_distributed_qa_with_rowless_q_ctas(built_lib, oracle_lib, write_model):
    """Head dim 128 over hidden 1280 takes the distributed QA form with only
    112 q / k / v tiles for the 148 CTAs, so some q CTAs own no rows of the
    projection and still attend (the shape of a 72B rank at TP8).  Context
    past two attention tiles; teacher-forced logits and greedy ids vs the
    oracle."""
    shape = gw.ModelShape("llama", 1280, 2, 10, 2, 1024, 1024, 512, 1e-5, 5e5, False, False, "q8_0", 1, 2)
    path = write_model("dist-qa-rowless", shape)
    m = b2decode.Model(path, num_ctx=512)
    g = goref.GoRef(path, num_ctx=512, n_threads=0)
    prompt = gw.make_prompt(shape.vocab, 150, seed=8)
    toks = np.concatenate([[shape.bos_id], prompt, gw.make_prompt(shape.vocab, 10, seed=9)]).astype(np.int32)
    pairs = teacher_forced(m.forward, g.forward, toks, 151)
    errs = [rel_l2(a, b) for a, b in pairs]
    assert max(errs) < LOGIT_TOL, errs
    assert np.mean([int(np.argmax(a)) == int(np.argmax(b)) for a, b in pairs]) >= 0.99
