"""The decode kernel's static work plans cover every weight tile exactly once.

tests/plan_check.cpp compiles the plan functions of csrc/dev.cuh (the same
code the producer warp, the consumer warps and the loader evaluate) as plain
C++ and checks, for every CTA of a 148-SM grid: each phase's tiles are split
over the grid exactly once, the residual rows go to the last CTAs, every
CTA's K-slices cover the blocks of a row with no empty slice, and every chunk
fits one ring slot; for the QA phase, for every split count in both the fused
and the distributed form.  The shapes are the measured models and, under
tensor parallelism, each rank's share (b2decode.tp.shares).
"""
import os
import subprocess

import pytest

from b2decode import tp

HERE = os.path.dirname(os.path.abspath(__file__))
GRID = 148  # B200 SMs: one decode CTA per SM

# (name, hidden, heads, kv_heads, ffn, vocab)
MODELS = [
    ("qwen2.5-0.5b", 896, 14, 2, 4864, 151936),
    ("llama3-8b", 4096, 32, 8, 14336, 128256),
    ("qwen2.5-72b", 8192, 64, 8, 29568, 152064),
    ("tp2-test", 1024, 8, 4, 1184, 1000),
    ("wide-heads", 2048, 16, 4, 5632, 32000),
]


@pytest.fixture(scope="module")
def plan_check(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("plans") / "plan_check")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I/usr/local/cuda/include", "-o", exe,
                    os.path.join(HERE, "plan_check.cpp")], check=True)
    return exe


def test_checker_reports_a_planted_error(plan_check):
    out = subprocess.run([plan_check, "selftest"], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout


def _cases():
    for name, h, nh, nkv, ff, v in MODELS:
        for deg in (1, 2, 4, 8):
            if nh % deg or nkv % deg:
                continue
            if deg > 1 and name in ("qwen2.5-0.5b",):
                continue
            for rank in sorted({0, deg - 1}):
                for qt in (8, 2):
                    yield pytest.param(name, h, nh, nkv, ff, v, deg, rank, qt, id=f"{name}-tp{deg}r{rank}-q{qt}")


@pytest.mark.parametrize("name,h,nh,nkv,ff,v,deg,rank,qt", list(_cases()))
def test_plans_cover_every_tile_once(plan_check, name, h, nh, nkv, ff, v, deg, rank, qt):
    s = tp.shares(h, nh, nkv, ff, v, deg, rank)
    hd = h // nh
    qd = s["q_rows"][1] - s["q_rows"][0]
    kvd = s["kv_rows"][1] - s["kv_rows"][0]
    ffl = s["ffn_rows"][1] - s["ffn_rows"][0]
    vl = s["vocab_rows"][1] - s["vocab_rows"][0]
    args = [h, qd, kvd, ffl, vl, nh // deg, hd, GRID, qt]
    out = subprocess.run([plan_check] + [str(a) for a in args], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", (args, out.stdout)
