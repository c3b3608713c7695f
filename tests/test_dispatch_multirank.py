"""Multi-rank (N > 1) host path on the CPU: request assignment, descriptor scatter, per-rank pools,
result gather and max-over-ranks timing, on two `gloo` ranks (tests/multirank_worker.py).

The data path has no collective: every request's output must come out of whichever rank ran it
exactly as a single process computes it. Each rank's pool must hold only its own requests, with
the same lowest-free-first block tables a single-rank pool gives for that request sequence."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import dispatch
from block_model import PoolModel

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import multirank_worker as W  # noqa: E402


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(tmp_path, world=2, extra=(), timeout=120):
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port()), WORLD_SIZE=str(world))
    procs = []
    for r in range(world):
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "multirank_worker.py"), "--out",
                                       str(tmp_path), *extra], env=dict(env, RANK=str(r)),
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append((p.returncode, out.decode(errors="replace")))
    return outs


def test_assign_balanced_and_modulo():
    lens = [700, 816, 750, 701, 802, 760, 799, 733, 790]
    for world in (1, 2, 3, 4):
        for policy in ("balanced", "modulo"):
            parts = dispatch.assign_requests(lens, world, policy)
            flat = sorted(i for p in parts for i in p)
            assert flat == list(range(len(lens)))
            assert max(len(p) for p in parts) <= -(-len(lens) // world)
    even = lens + [744]  # equal counts per rank: the key totals differ by less than one spread
    parts = dispatch.assign_requests(even, 2, "balanced")
    assert [len(p) for p in parts] == [5, 5]
    loads = [sum(even[i] for i in p) for p in parts]
    assert abs(loads[0] - loads[1]) <= max(even) - min(even)
    assert dispatch.assign_requests(lens, 3, "modulo")[1] == [1, 4, 7]
    with pytest.raises(ValueError):
        dispatch.assign_requests(lens, 0)


@pytest.mark.parametrize("policy", ["balanced", "modulo"])
def test_two_gloo_ranks_match_single_process(tmp_path, policy):
    outs = run_ranks(tmp_path, 2, ("--policy", policy))
    for rc, log in outs:
        assert rc == 0, log
    table = dispatch.make_requests(9, 5, 60, seed=7)
    parts = dispatch.assign_requests([r.prefix_len for r in table], 2, policy)
    res = np.load(tmp_path / "results.npz")
    assert float(res["max_t"]) == 2.0  # max over ranks of (rank + 1)
    np.testing.assert_array_equal(res["stacked"], np.stack([np.full((2, 3), 1.0), np.full((2, 3), 2.0)]))
    for r in table:  # every request once, identical to a single-process run
        np.testing.assert_array_equal(res[f"r{r.req_id}"], W.request_output(r))
    for rank in range(2):
        lines = (tmp_path / f"rank{rank}.txt").read_text().splitlines()
        assert [int(x) for x in lines[0].split()] == parts[rank]
        # the rank's pool, replayed by the allocation model over the same request order
        mine = [table[i] for i in parts[rank]]
        need = [(r.prefix_len + W.BT - 1) // W.BT for r in mine]
        model = PoolModel(n_blocks=sum(need), block_tokens=W.BT, max_seqs=len(mine), max_blocks_per_seq=max(need))
        for line, r in zip(lines[1:], mine):
            k, n, *blocks = (int(x) for x in line.split())
            s = model.seq_create()
            model.seq_resize(s, r.prefix_len)
            assert k == r.req_id and n == r.prefix_len
            assert blocks == model.seqs[s]["blocks"]


def test_rank_that_leaves_is_seen_by_the_other(tmp_path):
    outs = run_ranks(tmp_path, 2, ("--fail-rank", "1"), timeout=90)
    assert outs[1][0] == 3
    assert outs[0][0] != 0  # rank 0's gather ends with an error instead of waiting forever
    assert not (tmp_path / "results.npz").exists()
