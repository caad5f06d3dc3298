"""b2_matvec_batch (up to sixteen vectors per pass over W) against the oracle's
restatement of the Go Q8_0 / Q4_0 matvec, one vector at a time.

The kernel splits each vector into three int8 planes (about 22 bits relative
to the 32-block maximum), so its dots agree with the fp32 loop to rounding:
the bar is the batch-1 entry point's, 1e-5 relative L2 per vector.
"""
import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def _case(kind, rows, cols, nvec, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    raw = gw.quantize(w, gw.TYPE_NAMES[kind])
    x = rng.standard_normal((nvec, cols), dtype=np.float32)
    return raw, x


def _run(torch, kind, raw, x, rows, cols):
    nvec = x.shape[0]
    dw = torch.from_numpy(raw).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dy = torch.full((nvec, rows), float("nan"), device="cuda")
    b2decode.matvec_batch(8 if kind == "q8_0" else 2, dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols, nvec)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def _check(got, raw, x, rows, cols, kind, vecs):
    assert np.isfinite(got).all()
    for v in vecs:
        want = goref.matvec(kind, raw, x[v], rows, cols)
        assert rel_l2(got[v], want) < TOL, (v, rel_l2(got[v], want))


@pytest.mark.parametrize("kind", ["q8_0", "q4_0"])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)])
def test_config1_shapes_batch8(built_lib, oracle_lib, torch_cuda, kind, rows, cols):
    raw, x = _case(kind, rows, cols, 8, rows ^ cols)
    got = _run(torch_cuda, kind, raw, x, rows, cols)
    _check(got, raw, x, rows, cols, kind, (0, 7) if rows > 20000 else range(8))


@pytest.mark.parametrize("kind", ["q8_0", "q4_0"])
@pytest.mark.parametrize("rows,cols,nvec", [(17, 256, 3), (40, 512, 8), (33, 768, 5), (1000, 2048, 1), (16, 256, 2),
                                            (24, 512, 16), (17, 256, 12), (4096, 4096, 16), (300, 14336, 9)])
def test_ragged_rows_and_partial_batches(built_lib, oracle_lib, torch_cuda, kind, rows, cols, nvec):
    """Row counts off the 16-row tile, partial column tiles (fewer than 8, or
    9..16 vectors in two column tiles), and shapes small enough that the
    blocks are split into slices merged by the last unit of each tile."""
    raw, x = _case(kind, rows, cols, nvec, rows * 31 + cols + nvec)
    x[0, :32] *= 1e-3       # a block of tiny values
    if nvec > 2:
        x[2, 32:64] = 0.0   # an all-zero block
    got = _run(torch_cuda, kind, raw, x, rows, cols)
    _check(got, raw, x, rows, cols, kind, range(nvec))


@pytest.mark.parametrize("kind", ["q8_0", "q4_0"])
def test_calls_in_a_row_are_independent_and_deterministic(built_lib, oracle_lib, torch_cuda, kind):
    """The slice counters are reset by each call (a second split call, and one
    after an unsplit call, are still right) and equal inputs give equal bits."""
    shapes = [(300, 4096, 8), (128256, 4096, 8), (300, 4096, 8), (40, 512, 6), (300, 4096, 16), (40, 512, 6)]
    first = {}
    for i, (rows, cols, nvec) in enumerate(shapes):
        raw, x = _case(kind, rows, cols, nvec, 7 + rows)
        got = _run(torch_cuda, kind, raw, x, rows, cols)
        _check(got, raw, x, rows, cols, kind, (0, nvec - 1) if rows > 20000 else range(nvec))
        key = (rows, cols, nvec)
        if key in first:
            assert np.array_equal(first[key], got)
        first[key] = got


def test_batch1_agrees_with_b2_matvec(built_lib, oracle_lib, torch_cuda):
    torch = torch_cuda
    rows, cols = 4096, 4096
    raw, x = _case("q8_0", rows, cols, 1, 5)
    got = _run(torch, "q8_0", raw, x, rows, cols)[0]
    dw = torch.from_numpy(raw).cuda()
    dx = torch.from_numpy(x[0]).cuda()
    dy = torch.empty(rows, device="cuda")
    b2decode.matvec(8, dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    assert rel_l2(got, dy.cpu().numpy()) < 2 * TOL


MODEL_SHAPES = {
    "tiny-q8": gw.SHAPES["tiny"],
    "tiny-llama-q4": gw.SHAPES["tiny-llama-q4"],
    "wide-q4": gw.ModelShape("llama", 1024, 1, 8, 2, 2816, 1000, 256, 1e-5, 5e5, False, False, "q4_0", 1, 2),
    "wide-q8": gw.ModelShape("qwen2", 1024, 1, 8, 2, 2816, 1000, 256, 1e-6, 1e6, True, False, "q8_0", 1, 2),
}


@pytest.mark.parametrize("key", list(MODEL_SHAPES))
def test_model_matvec_over_resident_tiled_weights(built_lib, oracle_lib, torch_cuda, write_model, key):
    """b2_model_matvec reads the loader's tiled blocks: every projection of
    layer 0 (k and v start inside the fused QKV matrix), the embedding and
    the untied lm_head, against the dequantised tensor (bit-exact with the
    oracle) times x in float64."""
    torch = torch_cuda
    shape = MODEL_SHAPES[key]
    m = b2decode.Model(write_model(key, shape), num_ctx=64)
    H, qd, kvd, ff, V = shape.hidden, shape.hidden, shape.kv_dim, shape.ffn, shape.vocab
    dims = {"blk.0.attn_q.weight": (qd, H), "blk.0.attn_k.weight": (kvd, H), "blk.0.attn_v.weight": (kvd, H),
            "blk.0.attn_output.weight": (H, qd), "blk.0.ffn_down.weight": (H, ff), "token_embd.weight": (V, H)}
    if not shape.tied:
        dims["output.weight"] = (V, H)
    rng = np.random.default_rng(3)
    for name, (rows, cols) in dims.items():
        w = m.dequant(name, rows * cols).reshape(rows, cols).astype(np.float64)
        for nvec in (1, 8, 13):
            x = rng.standard_normal((nvec, cols), dtype=np.float32)
            dx = torch.from_numpy(x).cuda()
            dy = torch.full((nvec, rows), float("nan"), device="cuda")
            m.matvec(name, dx.data_ptr(), dy.data_ptr(), nvec)
            torch.cuda.synchronize()
            got = dy.cpu().numpy()
            want = x.astype(np.float64) @ w.T
            for v in range(nvec):
                assert rel_l2(got[v], want[v]) < TOL, (name, nvec, v, rel_l2(got[v], want[v]))
    x = torch.zeros((1, H), device="cuda")
    y = torch.zeros((1, ff), device="cuda")
    with pytest.raises(b2decode.B2Error) as e:
        m.matvec("blk.0.ffn_gate.weight", x.data_ptr(), y.data_ptr(), 1)
    assert e.value.code == -8
    m.close()
