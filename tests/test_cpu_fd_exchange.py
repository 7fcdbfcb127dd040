"""The descriptor exchange a tensor-parallel group runs before its peer-memory all-reduce
(host/src/fd_exchange.cpp): every rank sends its buffer's file descriptor to every other
rank over abstract Unix sockets and receives theirs. Host logic only, so it runs here as
real processes on the CPU (ordinary memory files stand in for the exported GPU buffers):
groups of 2 to 8 ranks, two successive exchanges of one group, and a rank that never
joins -- the others give up within their time limit, with nothing left open."""
import json
import os
import random
import subprocess
import tempfile
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC_DIR = os.path.join(ROOT, "qwen3.5-cpu-cpp_b200", "host", "src")
_BIN = None


def driver():
    global _BIN
    if _BIN is None:
        out = os.path.join(tempfile.mkdtemp(prefix="qwc_fdx_"), "fd_exchange_driver")
        subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", SRC_DIR,
                        os.path.join(ROOT, "tests", "cpp", "fd_exchange_driver.cpp"),
                        os.path.join(SRC_DIR, "fd_exchange.cpp"), "-o", out], check=True)
        _BIN = out
    return _BIN


def run_group(world, ranks=None, gen=1, timeout_ms=10000, group=None):
    """Starts `ranks` (default: all) of a group of `world` at once; their JSON lines."""
    group = group if group is not None else random.getrandbits(64)
    ranks = list(range(world)) if ranks is None else ranks
    procs = [subprocess.Popen([driver(), f"{group:x}", str(gen), str(r), str(world), str(timeout_ms)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in ranks]
    out = {}
    for r, p in zip(ranks, procs):
        so, _ = p.communicate(timeout=timeout_ms / 1000 + 30)
        out[r] = (p.returncode, json.loads(so.strip().splitlines()[-1]))
    return out


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_every_rank_receives_every_other_ranks_descriptor(world):
    res = run_group(world)
    for r, (rc, line) in res.items():
        assert rc == 0 and line["ok"], line
        assert sorted(int(q) for q in line["peers"]) == [q for q in range(world) if q != r]
        for q, (token, size) in line["peers"].items():
            assert token == f"token {q}"          # the peer's own memory file
            assert size == 1000 + int(q)          # and the size it announced
        assert line["fds_after"] == line["fds_before"]


def test_successive_exchanges_of_one_group():
    group = random.getrandbits(64)
    for gen in (1, 2):
        res = run_group(3, gen=gen, group=group)
        assert all(rc == 0 and line["ok"] for rc, line in res.values())


def test_a_rank_that_never_joins_makes_the_others_give_up_in_time():
    t0 = time.time()
    res = run_group(3, ranks=[0, 1], timeout_ms=1500)
    assert time.time() - t0 < 15.0
    for r, (rc, line) in res.items():
        assert rc == 1 and not line["ok"]
        assert "rank 2" in line["why"] or "did not arrive" in line["why"], line["why"]
        assert line["fds_after"] == line["fds_before"]


def test_invalid_group_arguments_are_refused():
    res = run_group(9, ranks=[0], timeout_ms=500)
    rc, line = res[0]
    assert rc == 1 and not line["ok"] and "2..8" in line["why"]
