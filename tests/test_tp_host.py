"""Tensor-parallel host logic on CPU: the shares each rank keeps and the
handle exchange between ranks (two gloo processes, world size 2)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import b2decode
from b2decode import tp


@pytest.mark.parametrize("source", ["loader", "restatement"])
def test_shares_cover_the_model_once(built_lib, source):
    """The loader's own share arithmetic (b2_tp_share_of, host only) and the
    Python restatement in b2decode.tp: each rank's slices, for the
    Qwen2.5-72B shape at TP 1/2/4/8."""
    # heads and vocab split evenly, the FFN at 32-element blocks (924 blocks
    # -> 116/115 at TP8, 3712/3680 rows)
    H, nh, nkv, FF, V = 8192, 64, 8, 29568, 152064
    share = b2decode.tp_share_of if source == "loader" else tp.shares
    for n in (1, 2, 4, 8):
        parts = [share(H, nh, nkv, FF, V, n, r) for r in range(n)]
        for key, total in (("q_rows", 64 * 128), ("kv_rows", 8 * 128), ("ffn_rows", FF), ("vocab_rows", V)):
            cur = 0
            for p in parts:
                a, b = p[key]
                assert a == cur and b > a
                cur = b
            assert cur == total, key
        for p in parts:
            assert p["wo_cols"] == p["q_rows"] and p["down_cols"] == p["ffn_rows"]
            assert (p["ffn_rows"][1] - p["ffn_rows"][0]) % 32 == 0
    sizes = sorted({p["ffn_rows"][1] - p["ffn_rows"][0] for p in (share(H, nh, nkv, FF, V, 8, r) for r in range(8))})
    assert sizes == [3680, 3712]


def test_restatement_matches_the_loader(built_lib):
    for shape in ((8192, 64, 8, 29568, 152064), (4096, 32, 8, 14336, 128256), (1024, 8, 4, 1184, 1000)):
        for n in (1, 2, 4, 8):
            if shape[1] % n or shape[2] % n:
                continue
            for r in range(n):
                assert b2decode.tp_share_of(*shape, n, r) == tp.shares(*shape, n, r), (shape, n, r)


def test_shares_reject_indivisible_heads(built_lib):
    with pytest.raises(ValueError):
        tp.shares(896, 14, 2, 4864, 151936, 4, 0)  # 2 KV heads over 4 ranks
    with pytest.raises(ValueError):
        tp.shares(896, 14, 2, 4864, 151936, 2, 2)
    for args in ((896, 14, 2, 4864, 151936, 4, 0), (896, 14, 2, 4864, 151936, 2, 2)):
        with pytest.raises(b2decode.B2Error) as e:
            b2decode.tp_share_of(*args)
        assert e.value.code == -8


class _FakeModel:
    """Stands in for a loaded rank: a rank-specific handle, records what
    connect passes back."""

    def __init__(self, rank):
        self.rank = rank
        self.got = None

    def tp_handle(self):
        return bytes([self.rank]) * 64

    def tp_connect(self, handles):
        self.got = handles


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = _FakeModel(rank)
        tp.connect(m)
        q.put((rank, [h[0] for h in m.got], [len(h) for h in m.got]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_handle_exchange_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank receives every rank's handle, in rank order
    assert res == [(0, [0, 1], [64, 64]), (1, [0, 1], [64, 64])]
