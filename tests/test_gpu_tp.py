"""Tensor-parallel decode on 2 GPUs (one process per GPU, peer stores over
NVLink): whole-vocabulary logits assembled from the ranks' shares and the
greedy ids against one GPU and against the oracle (skipped with fewer than
two GPUs).  On one GPU: every rank's share, loaded one rank after another,
decodes to its block of the whole tensor."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import b2decode
import goref
from b2decode import gguf_writer as gw

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("arch,wtype,bias", [("qwen2", "q8_0", True), ("llama", "q4_0", False)])
def test_tp2_matches_one_gpu_and_oracle(built_lib, oracle_lib, write_model, tmp_path, arch, wtype, bias):
    # 72B-like layout at a small size: 8 query / 4 KV heads of 128, uneven
    # FFN shares (37 blocks -> 18 / 19), vocab split in two
    shape = gw.ModelShape(arch, 1024, 2, 8, 4, 1184, 1000, 512, 1e-6, 1e6, bias, not bias, wtype, 1, 2)
    path = write_model(f"tp-{arch}-{wtype}", shape)
    out = tmp_path / "tp2.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", "29517", os.path.join(HERE, "tp_worker.py"), path, str(out)]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["status"] == 0
    # one GPU, same steps
    m = b2decode.Model(path, num_ctx=256)
    mode = goref.MODE_GGML_Q4 if wtype == "q4_0" else goref.MODE_GO
    g = goref.GoRef(path, num_ctx=256, n_threads=0, mode=mode)
    toks = np.concatenate([[1], gw.make_prompt(shape.vocab, 70, seed=5), gw.make_prompt(shape.vocab, 10, seed=6)])
    toks = toks.astype(np.int32)
    one = [m.forward(toks[:71])] + [m.forward([t]) for t in toks[71:]]
    ref = [g.forward(toks[:71])] + [g.forward([t]) for t in toks[71:]]
    for k, (a, b, c) in enumerate(zip(res["logits"], one, ref)):
        assert rel_l2(a, b) < 1e-2, (k, rel_l2(a, b))   # different summation order of Wo / down only
        assert rel_l2(a, c) < 1e-2, (k, rel_l2(a, c))
        assert int(np.argmax(a)) == int(np.argmax(c)), k
    m.reset()
    first = m.forward_argmax(toks[:71])
    assert res["greedy"] == [first] + m.decode_greedy(first, 12).tolist()


@pytest.mark.parametrize("wtype", ["q8_0", "q4_0"])
def test_rank_shares_decode_to_their_blocks(built_lib, oracle_lib, write_model, wtype):
    # Row shares (q, k, v, gate, up, lm_head) and column shares (Wo, down:
    # a window of every row, read from the file row by row) of 2- and 4-way
    # splits, loaded on one GPU without connecting the ranks; FFN shares
    # uneven (37 blocks -> 18 / 19 and 9 / 9 / 9 / 10).
    shape = gw.ModelShape("qwen2", 1024, 2, 8, 4, 1184, 1000, 512, 1e-6, 1e6, True, False, wtype, 1, 2)
    path = write_model(f"tp-shares-{wtype}", shape)
    mode = goref.MODE_GGML_Q4 if wtype == "q4_0" else goref.MODE_GO
    H, FF, V, hd = shape.hidden, shape.ffn, shape.vocab, shape.hidden // shape.heads
    dims = {"attn_q": (H, H), "attn_k": (shape.kv_heads * hd, H), "attn_v": (shape.kv_heads * hd, H),
            "attn_output": (H, H), "ffn_gate": (FF, H), "ffn_up": (FF, H), "ffn_down": (H, FF)}
    whole = {}
    for l in range(shape.layers):
        for k, (r, c) in dims.items():
            name = f"blk.{l}.{k}.weight"
            whole[name] = goref.dequant_tensor(path, name, r * c, mode=mode).reshape(r, c)
    whole["output.weight"] = goref.dequant_tensor(path, "output.weight", V * H, mode=mode).reshape(V, H)
    for tp in (2, 4):
        for rank in range(tp):
            sh = b2decode.tp_share_of(H, shape.heads, shape.kv_heads, FF, V, tp, rank)
            cut = {"attn_q": ("rows", sh["q_rows"]), "attn_k": ("rows", sh["kv_rows"]),
                   "attn_v": ("rows", sh["kv_rows"]), "attn_output": ("cols", sh["wo_cols"]),
                   "ffn_gate": ("rows", sh["ffn_rows"]), "ffn_up": ("rows", sh["ffn_rows"]),
                   "ffn_down": ("cols", sh["down_cols"])}
            m = b2decode.Model(path, num_ctx=64, tp_size=tp, tp_rank=rank)
            for l in range(shape.layers):
                for k, (axis, (a, b)) in cut.items():
                    name = f"blk.{l}.{k}.weight"
                    want = whole[name][a:b] if axis == "rows" else whole[name][:, a:b]
                    got = m.dequant(name, want.size).reshape(want.shape)
                    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(want).view(np.uint32)), \
                        (tp, rank, name)
            a, b = sh["vocab_rows"]
            got = m.dequant("output.weight", (b - a) * H).reshape(b - a, H)
            assert np.array_equal(got.view(np.uint32), whole["output.weight"][a:b].view(np.uint32)), (tp, rank)
            st = m.load_stats()
            m.close()
            # exactly the share's blocks (and the replicated embedding) crossed to the device:
            # Wo and down sent their column windows, not whole rows
            bpb = 34 if wtype == "q8_0" else 18
            q, kv, f = (np.diff(sh[k])[0] for k in ("q_rows", "kv_rows", "ffn_rows"))
            layer = (q + 2 * kv) * H + H * q + 2 * f * H + H * f
            want_bytes = (V * H + (b - a) * H + shape.layers * layer) // 32 * bpb
            assert st["bytes_uploaded"] == want_bytes, (tp, rank, st["bytes_uploaded"], want_bytes)
